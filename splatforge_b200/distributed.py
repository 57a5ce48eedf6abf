"""View-sharded data parallelism for training on a batch of views (one process per GPU).

The reference trains one view per step on one device (src/splatforge/studio/trainer.py:
218-248) and has no distributed code.  Here a step's batch of views is split across the
ranks of one node; the Gaussians are replicated; every rank renders its views forward
and backward through the B200 rasterizer, then the per-Gaussian parameter gradients are
summed across ranks with ONE all-reduce of a contiguous [N, 11 + 3K] float32 buffer
(means 3, log-scales 3, quaternion 4, opacity logit 1, SH 3K; 59 floats for SH degree
3) over NCCL (NVLink / NVSwitch), so that identical optimiser steps keep the replicas
in sync.

The rendering itself is independent per view, so no collective sits inside the
rasterizer; the all-reduce is ~2(n-1)/n * 236 MB per step for a million Gaussians.
"""

from __future__ import annotations

import datetime
import math
import os

import torch
import torch.distributed as dist

PARAM_ORDER = ("means", "log_scales", "quats", "opacity_logits", "sh")


def shard(items, rank, world):
    """Contiguous block partition of a batch of views: rank r gets items
    [r*len/world, (r+1)*len/world)."""
    n = len(items)
    lo, hi = rank * n // world, (rank + 1) * n // world
    return items[lo:hi]


def balanced_views(views, costs, world):
    """Cost-balanced assignment of one step's views to ``world`` ranks.

    ``views`` are view indices, ``costs[v]`` the measured render time of view v (the
    same table on every rank, see :func:`shared_view_costs`).  Longest processing time
    first: views in decreasing cost (ties by index) each go to the rank with the least
    load so far (ties to the lowest rank).  Ranks may get different numbers of views;
    the gradients are summed over all of them by the all-reduce either way, so the step
    computes the same sum while its slowest rank — the step's length in a synchronous
    step — carries as little as the costs allow.  Deterministic: every rank derives the
    same assignment.  Returns a list of ``world`` lists, each in increasing view order.
    """
    order = sorted(views, key=lambda v: (-float(costs[v]), v))
    load = [0.0] * world
    out = [[] for _ in range(world)]
    for v in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(v)
        load[r] += float(costs[v])
    return [sorted(o) for o in out]


def shared_view_costs(local_costs, n_views, device=None):
    """One cost table for every rank: ``local_costs`` maps the views this rank timed to
    their render times; the table holds, per view, the largest time any rank reported
    (0 for views no rank timed).  One all-reduce (MAX) of n_views floats when a process
    group is up."""
    t = torch.zeros(n_views, dtype=torch.float32, device=device)
    for v, c in local_costs.items():
        t[v] = max(float(t[v]), float(c))
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def query_shard(n, rank, shards):
    """[lo, hi) of query shard ``rank mod shards`` when ``n`` queries are cut into
    ``shards`` contiguous shards of sizes differing by at most one (the opacity-field
    workload: no collective, every rank evaluates its own queries)."""
    r = rank % shards
    return r * n // shards, (r + 1) * n // shards


def init_from_env(backend=None, timeout_s=120):
    """``torch.distributed`` from torchrun's RANK / WORLD_SIZE / LOCAL_RANK / MASTER_*.
    NCCL on CUDA (device bound to LOCAL_RANK), gloo otherwise.  A short timeout makes
    ranks that wait for a failed peer end with an error instead of hanging."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return rank, world, local
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, **kwargs)
    return rank, world, local


class GradientAllReduce:
    """Sums (or averages) the gradients of the Gaussian parameters across ranks with one
    collective on a packed [N, 11 + 3K] buffer.

    ``params`` is a sequence of the five parameter tensors in PARAM_ORDER (each [N, ...]).
    The packed buffer is allocated once and reused every step.

    With ``bind()`` the buffer is laid out parameter by parameter (means [N,3], then
    log-scales [N,3], quaternions [N,4], opacity logits [N], SH [N,3K]) and every
    parameter's ``.grad`` is a view of its block: autograd accumulates into the buffer in
    place, so the collective runs on the gradients where they already are, with no copy
    in or out.  ``zero_grad()`` clears the buffer at the start of a step.
    """

    def __init__(self, params, *, group=None, average=False, timed=False):
        self.params = list(params)
        if len(self.params) != len(PARAM_ORDER):
            raise ValueError("expected means, log_scales, quats, opacity_logits, sh")
        n = self.params[0].shape[0]
        if any(p.shape[0] != n for p in self.params):
            raise ValueError("all parameters must have the Gaussian count as their first dimension")
        self.widths = [math.prod(p.shape[1:]) for p in self.params]
        self.n = n
        self.group = group
        self.average = average
        self.buffer = torch.empty((n, sum(self.widths)), device=self.params[0].device, dtype=torch.float32)
        # with ``timed``: CUDA events (pack start, pack end, all-reduce end, unpack end)
        # recorded on the current stream around every call
        self.timed = timed
        self.events = []
        self.bound = False

    def bind(self):
        """Make every parameter's ``.grad`` a view of its block of the (flat) buffer."""
        flat = self.buffer.view(-1)
        col = 0
        self.views = []
        for p, w in zip(self.params, self.widths):
            v = flat[col * self.n:(col + w) * self.n].view(p.shape)
            self.views.append(v)
            col += w
        self.bound = True
        self.zero_grad()
        return self

    def zero_grad(self):
        """Zero the buffer and (re)attach the views as the parameters' gradients."""
        if not self.bound:
            for p in self.params:
                p.grad = None
            return
        self.buffer.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v

    def _in_place(self):
        return self.bound and all(
            p.grad is not None and p.grad.data_ptr() == v.data_ptr() for p, v in zip(self.params, self.views))

    @property
    def floats_per_gaussian(self):
        return sum(self.widths)

    def pack(self):
        lo, hi = self.buffer.data_ptr(), self.buffer.data_ptr() + self.buffer.numel() * self.buffer.element_size()
        # gradients that still alias the buffer (a bound reducer whose views were partly
        # replaced) are copied out before the buffer is overwritten
        grads = [None if p.grad is None else (p.grad.clone() if lo <= p.grad.data_ptr() < hi else p.grad)
                 for p in self.params]
        col = 0
        for g, w in zip(grads, self.widths):
            view = self.buffer[:, col : col + w]
            if g is None:
                view.zero_()
            else:
                view.copy_(g.reshape(self.n, w))
            col += w
        return self.buffer

    def unpack(self):
        col = 0
        for p, w in zip(self.params, self.widths):
            g = self.buffer[:, col : col + w].reshape(p.shape)
            if p.grad is None:
                p.grad = g.clone()
            else:
                p.grad.copy_(g)
            col += w

    def __call__(self):
        if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if self.timed else None
        in_place = self._in_place()
        if ev:
            ev[0].record()
        if not in_place:
            self.pack()
        if ev:
            ev[1].record()
        dist.all_reduce(self.buffer, op=dist.ReduceOp.SUM, group=self.group)
        if self.average:
            self.buffer /= dist.get_world_size(self.group)
        if ev:
            ev[2].record()
        if not in_place:
            self.unpack()
        if ev:
            ev[3].record()
            self.events.append(ev)

    def timings_ms(self):
        """Median (pack, all-reduce, unpack) milliseconds over the timed calls (after a
        synchronize), or None."""
        if not self.events:
            return None
        cols = list(zip(*[(a.elapsed_time(b), b.elapsed_time(c), c.elapsed_time(d)) for a, b, c, d in self.events]))
        return tuple(sorted(col)[len(col) // 2] for col in cols)
