"""View-sharded data parallelism on CPU ranks (gloo, world size 2).

The per-view renders are the CPU oracle's (these tests check the host-side
plumbing: sharding, packing of the [N, 59] gradient buffer, the all-reduce and the
failure behaviour), so no GPU is needed.
"""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import render as oracle_render
from splatforge_b200 import distributed, scenes

CH = ("rgb", "depth", "distortion_l1")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads_for(views, params, p=None):
    p = params.detach_clone().requires_grad_() if p is None else p
    for cam in views:
        out = oracle_render.render(scenes.activated(p), cam, mode="gof", distortions="l1")
        sum(out[c].sum() for c in CH).backward()
    return p


def _worker(rank, world, port, mode, queue):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        torch.set_num_threads(1)
        distributed.init_from_env(backend="gloo", timeout_s=10)
        params, cams = scenes.workload("demo48", seed=0)
        mine = distributed.shard(cams[:4], rank, world)
        if mode == "balanced":
            # each rank timed two of the four views; the shared table decides the split
            timed = {0: {0: 5.0, 1: 1.0}, 1: {2: 9.0, 3: 1.0}}[rank]
            costs = distributed.shared_view_costs(timed, 4)
            assert costs == [5.0, 1.0, 9.0, 1.0], costs
            split = distributed.balanced_views([0, 1, 2, 3], costs, world)
            assert split == [[2], [0, 1, 3]], split
            mine = [cams[i] for i in split[rank]]
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the all-reduce")
        if mode == "bound":
            # gradients accumulate straight into the collective's buffer
            p = params.detach_clone().requires_grad_()
            reducer = distributed.GradientAllReduce(p.tensors()).bind()
            _grads_for(mine, params, p)
            assert reducer._in_place()
        else:
            p = _grads_for(mine, params)
            reducer = distributed.GradientAllReduce(p.tensors())
        assert reducer.floats_per_gaussian == 59
        reducer()
        # numpy arrays travel by value: a torch tensor would be shared through a file
        # descriptor that dies with this process, racing the parent's read
        queue.put((rank, "ok", [t.grad.detach().cpu().numpy().copy() for t in p.tensors()]))
    except Exception as exc:  # report to the parent instead of hanging
        queue.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()[-400:]}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = {}
    for _ in procs:
        rank, status, payload = q.get(timeout=120)
        results[rank] = (status, payload)
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    return {r: (st, [torch.from_numpy(a) for a in pl] if st == "ok" else pl) for r, (st, pl) in results.items()}


def test_allreduced_gradients_equal_full_batch_gradients():
    res = _run("ok")
    assert all(s == "ok" for s, _ in res.values()), res
    params, cams = scenes.workload("demo48", seed=0)
    full = _grads_for(cams[:4], params)
    for rank in (0, 1):
        for got, want in zip(res[rank][1], full.tensors()):
            torch.testing.assert_close(got, want.grad, atol=2e-5, rtol=1e-4)


def test_gradients_bound_to_the_buffer_reduce_in_place():
    res = _run("bound")
    assert all(s == "ok" for s, _ in res.values()), res
    params, cams = scenes.workload("demo48", seed=0)
    full = _grads_for(cams[:4], params)
    for rank in (0, 1):
        for got, want in zip(res[rank][1], full.tensors()):
            torch.testing.assert_close(got, want.grad, atol=2e-5, rtol=1e-4)


def test_cost_balanced_views_sum_to_the_full_batch_gradients():
    """Ranks share their measured view costs, split the step's views longest first
    (one rank gets one view, the other three) and the all-reduce still yields the
    full batch's gradients on both."""
    res = _run("balanced")
    assert all(s == "ok" for s, _ in res.values()), res
    params, cams = scenes.workload("demo48", seed=0)
    full = _grads_for(cams[:4], params)
    for rank in (0, 1):
        for got, want in zip(res[rank][1], full.tensors()):
            torch.testing.assert_close(got, want.grad, atol=2e-5, rtol=1e-4)


def test_balanced_views_partition_and_bound():
    import random

    rnd = random.Random(3)
    for world in (1, 2, 3, 8):
        costs = [rnd.choice([1.0, 1.2, 0.9, 11.0]) for _ in range(64)]
        views = list(range(5, 5 + 8 * world))
        views = [v % 64 for v in views]
        split = distributed.balanced_views(views, costs, world)
        assert sorted(v for part in split for v in part) == sorted(views)
        assert split == distributed.balanced_views(views, costs, world)  # deterministic
        loads = [sum(costs[v] for v in part) for part in split]
        # longest-first greedy: within the largest single cost of the average, and never
        # worse than the round-robin blocks of 8
        total = sum(costs[v] for v in views)
        assert max(loads) <= total / world + max(costs[v] for v in views) + 1e-9
        blocks = [sum(costs[v] for v in views[8 * r:8 * r + 8]) for r in range(world)]
        assert max(loads) <= max(blocks) + 1e-9


def test_bound_views_and_fallback_packing_on_one_process():
    params, _ = scenes.workload("demo48", seed=0)
    p = params.detach_clone().requires_grad_()
    r = distributed.GradientAllReduce(p.tensors()).bind()
    flat = r.buffer.view(-1)
    offset = 0
    for t in p.tensors():
        assert t.grad.data_ptr() == flat[offset:].data_ptr() and t.grad.shape == t.shape
        offset += t.numel()
    assert offset == flat.numel() and float(flat.abs().sum()) == 0.0
    # a replaced gradient: packing copies every gradient, aliasing ones included
    for k, t in enumerate(p.tensors()):
        t.grad.fill_(k + 1.0)
    p.means.grad = torch.full_like(p.means, 7.0)
    assert not r._in_place()
    buf = r.pack().clone()
    col = 0
    for k, (t, w) in enumerate(zip(p.tensors(), r.widths)):
        want = 7.0 if k == 0 else k + 1.0
        assert torch.all(buf[:, col:col + w] == want)
        col += w


def test_query_shards_partition_the_query_set():
    for n, shards in ((20_000_001, 8), (7, 8), (0, 8), (1000, 3)):
        spans = [distributed.query_shard(n, r, shards) for r in range(shards)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [hi - lo for lo, hi in spans]
        assert max(sizes) - min(sizes) <= 1
    # more ranks than shards: rank r evaluates shard r mod shards
    assert distributed.query_shard(100, 9, 8) == distributed.query_shard(100, 1, 8)


def test_failed_rank_ends_its_peer_with_an_error_not_a_hang():
    res = _run("fail")
    assert res[1][0] == "error" and "rank 1 failed" in res[1][1]
    assert res[0][0] == "error", "the surviving rank must see an error from the collective"


def test_shard_partitions_views():
    views = list(range(10))
    parts = [distributed.shard(views, r, 4) for r in range(4)]
    assert sum(parts, []) == views
    assert max(map(len, parts)) - min(map(len, parts)) <= 1
