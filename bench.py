"""Forward + backward throughput of the B200 rasterizer (Mpix/s), 1..8 GPUs.

Workload (default): the 1M-Gaussian surface scene at 1920x1080, 60 deg FOV,
GOF mode with the full distortion set ("both": RGB, expected depth, median depth,
normal, L1 and L2 distortion, ray colour, ambiguity) forward + backward against
fixed seeded upstream gradients on every output.  Each rank renders its own view
of the replicated scene per step; with N > 1 ranks the per-Gaussian gradients
(59 floats per Gaussian) are all-reduced with NCCL every step (view-sharded data
parallelism).  ``value`` = all ranks' rendered pixels / max-over-ranks step time.

``--workload surfaces3m_views64`` runs the view-batched training step instead: 3M
Gaussians, 8 views of 1600x1064 per GPU per step (8/16/32/64 views at 1/2/4/8 GPUs),
gradients accumulated over the views, then one all-reduce of the [N,59] buffer.
``--workload field2m_views32`` times the GOF opacity field (queries/s) and
``--workload mesh100k_views32`` the GOF mesh extraction (tetrahedra/s).

    python bench.py [--gpus N --steps K --warmup W]          # B200 arm
    python bench.py --impl reference [...]                     # CPU arm (oracle port)
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CHANNELS = ("rgb", "alpha", "depth", "normals", "distortion_l1", "distortion_l2",
            "median_depth", "ray_color", "ambiguity_mask")
METRIC = "fwd+bwd rendered Mpix/s at 1M Gaussians 1080p; views/s at 1/2/4/8 GPUs"
# workloads rendered as a batch of views per GPU per step (the rest: one view)
VIEW_BATCHED = {"surfaces3m_views64": 8}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", default="surfaces1m_1080p")
    ap.add_argument("--mode", default="gof")
    ap.add_argument("--distortions", default="both")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._proc = None

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return self

        def reader():
            for line in self._proc.stdout:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 7:
                    self.samples.append(parts)

        self._t = threading.Thread(target=reader, daemon=True)
        self._t.start()
        return self

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        sm = []
        reasons = set()
        maxmhz = None
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for s in self.samples:
            try:
                sm.append(float(s[0]))
                maxmhz = float(s[1])
            except ValueError:
                continue
            for name, flag in zip(names, s[3:]):
                if flag.lower() == "active":
                    reasons.add(name)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": maxmhz, "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant
# kernel, from a single-pass ncu capture of this exact workload.
MEASURED_TRAFFIC = {("surfaces1m_1080p", "gof", "both", "raster_backward"): 3212488192 + 73037056}


def algorithmic_flops(mode, n_pairs_fwd):
    """Per-pair algorithmic FP32 flops of the raster forward: the sample equations of
    each mode (GOF: Q r, the ray peak, the offset, its quadratic form, the normal)."""
    per = {"radegs": 35, "gof": 70, "ambisur": 40}[mode]
    return per * n_pairs_fwd


def run_b200(args):
    import torch.distributed as dist

    from splatforge_b200 import distributed, rasterizer, scenes
    from splatforge_b200.renderer import B200Renderer
    from splatforge_b200.rasterizer import RasterSettings

    rank, world, local = distributed.init_from_env(backend="nccl", timeout_s=300)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    params, wl_cams = scenes.workload(args.workload, seed=0)
    if args.workload in VIEW_BATCHED:
        # view-batched training step: VIEW_BATCHED views per GPU per step, drawn in
        # order from the workload's 64 poses (8/16/32/64 views at 1/2/4/8 GPUs)
        per = VIEW_BATCHED[args.workload]
        my_cams = [wl_cams[(rank * per + v) % len(wl_cams)] for v in range(per)]
    else:
        base_cam = wl_cams[0]
        cams = scenes.orbit_cameras(max(8, world), base_cam.width, base_cam.height,
                                    60.0 if "1080" in args.workload else 50.0, radius=3.0, seed=0)
        my_cams = [cams[0] if world == 1 else cams[rank]]
    cam = my_cams[0]
    settings = RasterSettings(mode=args.mode, distortions=args.distortions)
    g = torch.Generator().manual_seed(1234 + rank)
    H, W = cam.height, cam.width
    ups = {ch: torch.randn(H, W, 3 if ch in ("rgb", "normals") else 1, generator=g).to(dev) for ch in CHANNELS}
    p = params.to(dev).requires_grad_()
    n = p.means.shape[0]
    reducer = distributed.GradientAllReduce(p.tensors())

    prof = {"fwd": [], "bwd": []}

    def step(timing=False):
        for t in p.tensors():
            t.grad = None
        for c in my_cams:
            view = scenes.activated(p)
            out = rasterizer.rasterize(view.means, view.quats, view.scales, view.opacities, view.sh, 3, c, settings)
            loss = sum((out[ch] * ups[ch]).sum() for ch in CHANNELS)
            loss.backward()
        reducer()
        return out

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    n_isect = out["n_isect"]
    # per-kernel durations of the dominant kernels, on the launching stream
    rasterizer.PROFILE = prof
    launches0 = rasterizer.kernel_launches()
    clocks = ClockSampler(local).start() if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    rasterizer.PROFILE = None
    launches = rasterizer.kernel_launches() - launches0
    clk = clocks.stop() if clocks else None
    fwd_times = [a.elapsed_time(b) for a, b in prof["fwd"]]
    bwd_times = [a.elapsed_time(b) for a, b in prof["bwd"]]
    counters = prof["counters"][-1].tolist() if prof.get("counters") else [0, 0]
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    pixels = H * W * len(my_cams) * world
    value = pixels / (ms * 1e-3) / 1e6

    # end to end through the public renderer API: pinned host parameters in, loss out.
    # Every step uploads its parameters; the upload of step k+1 runs on a copy stream
    # into the second of two parameter buffers while step k renders (a prefetching
    # loader), and every upload lies inside the timed region.
    e2e = None
    if not args.no_e2e:
        renderer = B200Renderer(settings_config(settings), mode=args.mode)
        host = [t.detach().cpu().pin_memory() for t in params.tensors()]
        bufs = [[torch.empty_like(t, device=dev) for t in host] for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in host)
        loss_host = torch.empty((), pin_memory=True)
        reducers = [distributed.GradientAllReduce(b) for b in bufs]
        copy_stream = torch.cuda.Stream(device=dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]

        def upload(slot, after):
            with torch.cuda.stream(copy_stream):
                if after is not None:
                    copy_stream.wait_event(after)
                for d, h in zip(bufs[slot], host):
                    d.copy_(h, non_blocking=True)
                ready[slot].record(copy_stream)

        def e2e_steps(count, start):
            upload(0, start)
            for k in range(count):
                slot = k % 2
                torch.cuda.current_stream().wait_event(ready[slot])
                if k + 1 < count:
                    upload(1 - slot, freed[1 - slot] if k >= 1 else None)
                dev_params = bufs[slot]
                for d in dev_params:
                    d.requires_grad_(True)
                    d.grad = None
                sp = scenes.SceneParams(*dev_params, sh_degree=3)
                total = 0.0
                for c in my_cams:
                    v = scenes.activated(sp)
                    o = renderer.render(v, c, distortions=args.distortions)
                    loss = sum((getattr(o, ch) * ups[ch]).sum() for ch in CHANNELS)
                    loss.backward()
                    total = total + loss.detach()
                reducers[slot]()
                loss_host.copy_(total, non_blocking=True)
                for d in dev_params:
                    d.requires_grad_(False)
                freed[slot].record()

        e2e_steps(2, None)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        e2e_steps(args.steps, a0)
        a1.record()
        torch.cuda.synchronize()
        ems = a0.elapsed_time(a1) / args.steps
        te = torch.tensor([ems], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        ems = float(te.item())
        e2e = {"value": round(pixels / (ems * 1e-3) / 1e6, 3), "unit": "Mpix/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "ms_per_step": round(ems, 3),
               "upload": "pinned host -> device every step, overlapped with the previous step's render"}

    result = None
    if rank == 0:
        fwd = sorted(fwd_times)[len(fwd_times) // 2] if fwd_times else None
        bwd = sorted(bwd_times)[len(bwd_times) // 2] if bwd_times else None
        peaks = measured_peaks()
        sm_mhz = (clk or {}).get("sm_mhz") or 1965.0
        fp32_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
        roof = None
        if bwd is not None:
            dom, dom_ms = ("raster_backward", bwd) if bwd >= (fwd or 0) else ("raster_forward", fwd)
            pairs = counters[0]
            flops = algorithmic_flops(args.mode, pairs) * (2 if dom == "raster_backward" else 1)
            achieved = flops / (dom_ms * 1e-3) / 1e12
            roof = {"bound": "fp32", "kernel": dom, "achieved": round(achieved, 3),
                    "peak": round(fp32_peak, 2), "unit": "TFLOP/s", "frac": round(achieved / fp32_peak, 4),
                    "traffic": MEASURED_TRAFFIC.get((args.workload, args.mode, args.distortions, dom)),
                    "traffic_unit": "bytes per launch", "kernel_ms": round(dom_ms, 4),
                    "peak_source": f"FP32 SIMT 148 SM x 128 lanes x 2 at the sampled {sm_mhz:.0f} MHz",
                    "hbm_peak_gbs": peaks.get("hbm_gbs")}
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": "Mpix/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded surface-sampled scene, random camera poses)",
            "config": {"workload": f"{args.workload}: {n} Gaussians, {W}x{H}, mode {args.mode}, "
                                   f"distortions {args.distortions}, fwd+bwd, {len(my_cams)} view(s) per GPU per step",
                       "parallelism": f"view-sharded dp{world}, NCCL all-reduce of [N,59] grads" if world > 1 else "single GPU",
                       "views_per_s": round(world * len(my_cams) / (ms * 1e-3), 3), "n_isect": int(n_isect),
                       "l2_policy": "inputs larger than L2 (236 MB parameters + records per step)",
                       "fwd_ms": fwd, "bwd_ms": bwd, "pairs_evaluated": counters[0],
                       "pairs_contributing": counters[1], "pairs_in_tile_lists": int(n_isect) * 256},
            "gpu_launches": int(launches),
            "clocks": clk, "e2e": e2e, "roofline": roof,
        }
        # the CPU baseline is timed once, at N=1 (other ranks would compete for the cores)
        result["cpu_baseline"] = cpu_baseline(args) if world == 1 and not args.no_cpu_baseline else None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


FIELD_WORKLOADS = {"field2m_views32"}
FIELD_SHARDS = 8  # the query set is cut into 8 shards; rank r evaluates shard r


def run_field(args):
    """GOF opacity field over an extraction grid (9 points per Gaussian + 2M uniform),
    2M Gaussians, 32 view origins; each rank evaluates one eighth of the ~20M queries
    (weak scaling: 8 shards at 8 GPUs), no collective on the data path."""
    import torch.distributed as dist

    from splatforge_b200 import distributed, ops, scenes

    rank, world, local = distributed.init_from_env(backend="nccl", timeout_s=300)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    params, cams = scenes.workload(args.workload, seed=0)
    view = scenes.activated(params)
    queries = scenes.field_queries(params, 2_000_000, seed=0)
    q = queries.shape[0]
    lo, hi = (rank % FIELD_SHARDS) * q // FIELD_SHARDS, (rank % FIELD_SHARDS + 1) * q // FIELD_SHARDS
    host = {"pts": queries[lo:hi].contiguous().pin_memory(), "means": view.means.contiguous().pin_memory(),
            "Q": scenes.inverse_covariances(params).contiguous().pin_memory(),
            "opac": view.opacities.contiguous().pin_memory(),
            "origins": torch.stack([c.origin for c in cams]).contiguous().pin_memory()}
    d = {k: v.to(dev) for k, v in host.items()}
    n_q = hi - lo

    def step():
        return ops.opacity_field_culled(d["pts"], d["means"], d["Q"], d["opac"], d["origins"])

    launches0 = None
    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    from splatforge_b200 import rasterizer

    launches0 = rasterizer.kernel_launches()
    clocks = ClockSampler(local).start() if rank == 0 else None
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = step()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks else None
    launches = rasterizer.kernel_launches() - launches0
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = n_q * world / (ms * 1e-3)

    # end to end: queries and scene from pinned host memory in, field values out
    field_host = torch.empty((n_q,), pin_memory=True)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    a0.record()
    for _ in range(args.steps):
        for k, v in host.items():
            d[k].copy_(v, non_blocking=True)
        field_host.copy_(step(), non_blocking=True)
    a1.record()
    torch.cuda.synchronize()
    te = torch.tensor([a0.elapsed_time(a1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    ems = float(te.item())
    result = None
    if rank == 0:
        result = {
            "metric": "GOF opacity-field queries/s (2M Gaussians, 32 views)", "value": round(value, 1),
            "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded surface-sampled scene, exporter-shaped query grid)",
            "config": {"workload": f"{args.workload}: {params.means.shape[0]} Gaussians, {len(cams)} origins, "
                                   f"{n_q} queries per GPU ({q} in {FIELD_SHARDS} shards)",
                       "parallelism": f"query-sharded x{world}, no collective" if world > 1 else "single GPU",
                       "path": "culled per-view cube-map candidate lists (contributions <= 1e-7 dropped)",
                       "field_mean": round(float(out.mean().item()), 6)},
            "gpu_launches": int(launches), "clocks": clk,
            "e2e": {"value": round(n_q * world / (ems * 1e-3), 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(n_q * 4), "ms_per_step": round(ems, 3)},
            "roofline": None, "cpu_baseline": field_cpu_baseline(host) if world == 1 and not args.no_cpu_baseline else None,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def field_cpu_baseline(host, budget_s=15.0):
    """The oracle's field (the reference's brute-force restatement) on the host cores: a
    growing number of (query, origin) pairs (queries from this rank, one origin at a time)
    until the budget is used; its cost is linear in both, so the rate of pairs divided by
    the origin count gives queries/s over all origins."""
    from oracle import ops as oracle_ops

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    pts, m, Q, o, org = (host[k] for k in ("pts", "means", "Q", "opac", "origins"))
    pairs, spent, count, v = 0, 0.0, 2, 0
    while spent < budget_s:
        t0 = time.perf_counter()
        oracle_ops.opacity_field(pts[:count], m, Q, o, org[v % org.shape[0]:v % org.shape[0] + 1], gaussian_chunk=65536)
        spent += time.perf_counter() - t0
        pairs += count
        v += 1
        count = min(count * 2, 64)
    rate = pairs / spent / org.shape[0] if spent > 0 else 0.0
    return {"value": round(rate, 4), "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"oracle opacity field on {pairs} (query, origin) pairs ({spent:.1f} s) against all "
                      f"{m.shape[0]} Gaussians; linear in queries and origins, scaled to {org.shape[0]} origins"}


MESH_WORKLOADS = {"mesh100k_views32"}


class MeshJob:
    """GOF level-set extraction of the exporter (src/splatforge/studio/exporters.py:41-88)
    on a fixed tetrahedral grid: the seed Gaussians' grid and its Delaunay cells are built
    once (host Qhull, untimed); a step builds the culled field plan (every view's
    candidate lists), evaluates the field at every grid point and runs marching
    tetrahedra with 8 bisection steps (8 more field evaluations over the crossing edges)
    to the vertices and faces."""

    def __init__(self, workload, dev):
        from splatforge_b200 import meshing, scenes

        params, cams = scenes.workload(workload, seed=0)
        view = scenes.activated(params)
        self.n = params.means.shape[0]
        self.host = {"means": view.means.contiguous().pin_memory(), "quats": view.quats.contiguous().pin_memory(),
                     "scales": view.scales.contiguous().pin_memory(),
                     "opac": view.opacities.contiguous().pin_memory(),
                     "Q": scenes.inverse_covariances(params).contiguous().pin_memory(),
                     "origins": torch.stack([c.origin for c in cams]).contiguous().pin_memory()}
        self.d = {k: v.to(dev) for k, v in self.host.items()}
        t0 = time.perf_counter()
        points, cells, self.seeds = meshing.gaussian_grid(self.d["means"], self.d["quats"], self.d["scales"],
                                                          self.d["opac"])
        self.grid_seconds = time.perf_counter() - t0
        self.points_host, self.cells_host = points, cells
        self.points = torch.as_tensor(points, device=dev)
        self.cells = torch.as_tensor(cells, device=dev).to(torch.int32)
        self.queries = 0
        self.meshing = meshing

    def field(self, coordinates):
        self.queries += coordinates.shape[0]
        return self.plan(coordinates.to(torch.float32).contiguous())

    def step(self):
        from splatforge_b200 import ops

        d = self.d
        self.plan = ops.OpacityFieldPlan(d["means"], d["Q"], d["opac"], d["origins"])
        return self.meshing.marching_tetrahedra(self.points, self.cells, self.field(self.points), self.field,
                                                level=0.5, binary_steps=8)


def run_mesh(args):
    """Replicas: every rank extracts the same level set (the extraction's bisection
    steps depend on each other's results, so the path does not shard); value = ranks x
    tetrahedra / max-over-ranks step time."""
    import torch.distributed as dist

    from splatforge_b200 import distributed, rasterizer

    rank, world, local = distributed.init_from_env(backend="nccl", timeout_s=600)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    job = MeshJob(args.workload, dev)
    for _ in range(args.warmup):
        verts, faces = job.step()
    torch.cuda.synchronize()
    launches0 = rasterizer.kernel_launches()
    job.queries = 0
    clocks = ClockSampler(local).start() if rank == 0 else None
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        verts, faces = job.step()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks else None
    launches = rasterizer.kernel_launches() - launches0
    queries = job.queries // args.steps
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    n_cells = job.cells.shape[0]

    # end to end: the scene and the grid from pinned host memory, the mesh back to the host
    pts_pinned = job.points.cpu().pin_memory()
    cells_pinned = job.cells.cpu().pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in job.host.values()) + pts_pinned.numel() * 8 + cells_pinned.numel() * 4
    d2h = 0
    if world > 1:
        dist.barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(args.steps):
        for k, v in job.host.items():
            job.d[k].copy_(v, non_blocking=True)
        job.points.copy_(pts_pinned, non_blocking=True)
        job.cells.copy_(cells_pinned, non_blocking=True)
        verts, faces = job.step()
        vh, fh = verts.cpu(), faces.cpu()
        d2h = vh.numel() * 8 + fh.numel() * 8
    a1.record()
    torch.cuda.synchronize()
    te = torch.tensor([a0.elapsed_time(a1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    ems = float(te.item())
    result = None
    if rank == 0:
        result = {
            "metric": "GOF mesh extraction tetrahedra/s (100k Gaussians, 32 views, 8 bisection steps)",
            "value": round(n_cells * world / (ms * 1e-3), 1), "unit": "tetrahedra/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64 (grid, bisection) / f32 (field)",
            "data": "synthetic (seeded surface-sampled scene, exporter grid)",
            "config": {"workload": f"{args.workload}: {job.n} Gaussians ({job.seeds} seeds), "
                                   f"{len(job.points_host)} grid points, {n_cells} tetrahedra, "
                                   f"{job.d['origins'].shape[0]} origins, level 0.5",
                       "parallelism": f"{world} replicas" if world > 1 else "single GPU",
                       "field_queries_per_step": int(queries), "vertices": int(verts.shape[0]),
                       "faces": int(faces.shape[0]),
                       "untimed_setup": f"grid points (device) + dedup and Delaunay (host Qhull) "
                                        f"{job.grid_seconds:.1f} s"},
            "gpu_launches": int(launches), "clocks": clk,
            "e2e": {"value": round(n_cells * world / (ems * 1e-3), 1), "unit": "tetrahedra/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ems, 3)},
            "roofline": None,
            "cpu_baseline": mesh_cpu_baseline(job) if world == 1 and not args.no_cpu_baseline else None,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def mesh_cpu_baseline(job, field_budget_s=10.0):
    """The oracle on the host cores: its marching tetrahedra over the full grid, timed
    with the field values replayed from the device run (the oracle's bisection points
    are the device's, bit for bit), plus the oracle field's measured cost per query
    times the queries one extraction evaluates."""
    import numpy as np

    from oracle import meshing as oracle_meshing

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    recorded = []

    def record(c):
        v = job.field(c)
        recorded.append(v.double().cpu().numpy())
        return v

    job.meshing.marching_tetrahedra(job.points, job.cells, record(job.points), record, level=0.5, binary_steps=8)
    replay = iter(recorded[1:])
    t0 = time.perf_counter()
    oracle_meshing.marching_tetrahedra(job.points_host, job.cells_host, recorded[0], lambda p: next(replay),
                                       level=0.5, binary_steps=8)
    marching_s = time.perf_counter() - t0
    n_queries = sum(len(r) for r in recorded)
    field = field_cpu_baseline({"pts": job.points.float().cpu(), "means": job.host["means"], "Q": job.host["Q"],
                                "opac": job.host["opac"], "origins": job.host["origins"]}, budget_s=field_budget_s)
    field_s = n_queries / field["value"] if field["value"] else float("inf")
    total = marching_s + field_s
    return {"value": round(job.cells.shape[0] / total, 3), "unit": "tetrahedra/s", "cores": threads, "kind": "port",
            "sample": f"oracle marching over all {job.cells.shape[0]} tetrahedra ({marching_s:.1f} s, field values "
                      f"replayed) + oracle field at {field['value']:.2f} queries/s x {n_queries} queries "
                      f"({field_s:.0f} s, extrapolated from {field['sample']})"}


def settings_config(settings):
    from types import SimpleNamespace

    return SimpleNamespace(sigma_extent=settings.sigma_extent, eps2d=settings.eps2d, near=settings.near,
                           far=settings.far, background=settings.background, antialiased=settings.antialiased,
                           tile_size=settings.tile_size)


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


class CpuSample:
    """The oracle (CPU restatement of the Torch provider's renderer) on the same view,
    timed in three parts that add up to its full-frame fwd+bwd time:

    * ``prep``: projection, conics, colours and exact tile lists of all Gaussians
      (timed once, forward),
    * ``tiles``: forward + backward of uniformly sampled tile batches (padded, as the
      Torch provider batches them) down to the projected per-Gaussian tensors; the
      frame's tile time is the batch count times the mean,
    * ``prep_bwd``: the backward from the projected tensors to the parameters (once).
    """

    def __init__(self, args, threads):
        from oracle import render as oracle_render
        from splatforge_b200 import scenes

        torch.set_num_threads(threads)
        self.threads = threads
        self.render = oracle_render
        params, cams = scenes.workload(args.workload, seed=0)
        self.cam = cams[0]
        self.leaves = params.detach_clone().requires_grad_()
        t0 = time.perf_counter()
        view = scenes.activated(self.leaves)
        self.ctx = oracle_render.prepare(view, self.cam, mode=args.mode, distortions=args.distortions)
        self.t_prep = time.perf_counter() - t0
        names = ("xy", "conic", "colors", "ray_colors", "opacity", "m", "normals", "gain", "qinv", "plane")
        self.inter = [self.ctx[k] for k in names if self.ctx[k].requires_grad]
        g = torch.Generator().manual_seed(7)
        ups = [torch.randn(t.shape, generator=g) for t in self.inter]
        t0 = time.perf_counter()
        torch.autograd.grad(self.inter, self.leaves.tensors(), grad_outputs=ups, retain_graph=True, allow_unused=True)
        self.t_prep_bwd = time.perf_counter() - t0
        # tiles are timed against detached copies of the projected tensors, so that a
        # tile's backward stops there (the shared projection graph runs once, above)
        self.inter = []
        for k in names:
            t = self.ctx[k]
            if t.requires_grad:
                leaf = t.detach().requires_grad_()
                if hasattr(t, "absgrad"):
                    leaf.absgrad = torch.zeros_like(leaf)
                self.ctx[k] = leaf
                self.inter.append(leaf)
        self.batches = oracle_render.tile_batches(self.ctx)
        self.up = torch.randn(256, sum(c for _, c in oracle_render.CHANNELS), generator=g)

    def tiles(self, budget_s, rng):
        """Fwd+bwd seconds of uniformly sampled tile batches until ``budget_s`` is used."""
        times, spent = [], 0.0
        while spent < budget_s:
            tiles, longest = self.batches[int(rng.integers(len(self.batches)))]
            c0 = time.perf_counter()
            out = self.render.render_batch(self.ctx, tiles, longest)
            loss = (out * self.up[: out.shape[1]]).sum()
            if loss.requires_grad:
                torch.autograd.grad(loss, self.inter, allow_unused=True)
            dt = time.perf_counter() - c0
            times.append(dt)
            spent += dt
        return times

    def frame_seconds(self, times):
        return self.t_prep + len(self.batches) * (sum(times) / len(times)) + self.t_prep_bwd

    def describe(self, times):
        return (f"oracle fwd+bwd of {len(times)} uniformly sampled tile batches (of {len(self.batches)}, "
                f"formed as the Torch provider forms them) of the {self.cam.width}x{self.cam.height} view "
                f"({sum(times):.1f} s, mean {1e3 * sum(times) / len(times):.1f} ms/batch), plus the "
                f"full-scene projection/binning ({self.t_prep:.1f} s) and its backward "
                f"({self.t_prep_bwd:.1f} s), timed once")


def cpu_baseline(args, budget_s=20.0):
    import numpy as np

    threads = os.cpu_count() or 1
    try:
        sampler = CpuSample(args, threads)
        times = sampler.tiles(budget_s, np.random.default_rng(0))
        mpix = sampler.cam.width * sampler.cam.height / sampler.frame_seconds(times) / 1e6
    except Exception as exc:  # the baseline must not hide the GPU result
        return {"value": None, "unit": "Mpix/s", "cores": threads, "kind": "port", "sample": f"failed: {exc}"}
    return {"value": round(mpix, 6), "unit": "Mpix/s", "cores": threads, "kind": "port",
            "sample": sampler.describe(times)}


def run_reference(args):
    """The reference arm: the oracle port on the host cores, one bounded tile sample
    per step (about 3 s), each extrapolated to a full frame; value = median."""
    import numpy as np

    rank, world, _ = dist_env()
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    sampler = CpuSample(args, threads)
    rng = np.random.default_rng(0)
    for _ in range(args.warmup):
        sampler.tiles(0.5, rng)
    vals, all_times = [], []
    for _ in range(args.steps):
        times = sampler.tiles(3.0, rng)
        all_times += times
        vals.append(sampler.cam.width * sampler.cam.height / sampler.frame_seconds(times) / 1e6)
    wall = time.perf_counter() - t0
    value = sorted(vals)[len(vals) // 2]
    ms = sampler.frame_seconds(all_times) * 1e3
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "Mpix/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded surface-sampled scene)",
        "config": {"workload": f"{args.workload}: mode {args.mode}, distortions {args.distortions}, fwd+bwd, "
                               f"1 view per step", "wall_seconds": round(wall, 1)},
        "cpu_baseline": {"value": round(value, 6), "unit": "Mpix/s", "cores": threads, "kind": "port",
                         "sample": sampler.describe(all_times)},
        "e2e": {"value": round(value, 6), "unit": "Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference_field(args):
    """The reference arm of the field workload: the oracle field on the host cores, one
    bounded (query, origin) sample per step; value = median rate."""
    from splatforge_b200 import scenes

    rank, world, _ = dist_env()
    if rank != 0:
        return None
    params, cams = scenes.workload(args.workload, seed=0)
    view = scenes.activated(params)
    host = {"pts": scenes.field_queries(params, 2_000_000, seed=0)[:4096], "means": view.means,
            "Q": scenes.inverse_covariances(params), "opac": view.opacities,
            "origins": torch.stack([c.origin for c in cams])}
    for _ in range(args.warmup):
        field_cpu_baseline(host, budget_s=0.5)
    runs = [field_cpu_baseline(host, budget_s=5.0) for _ in range(args.steps)]
    value = sorted(r["value"] for r in runs)[len(runs) // 2]
    return {"impl": "reference", "metric": "GOF opacity-field queries/s (2M Gaussians, 32 views)", "value": value,
            "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 / value, 1) if value else None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded surface-sampled scene)",
            "config": {"workload": f"{args.workload}: {params.means.shape[0]} Gaussians, {len(cams)} origins"},
            "cpu_baseline": {**runs[len(runs) // 2], "value": value},
            "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    if args.impl == "reference" and args.workload in FIELD_WORKLOADS:
        res = run_reference_field(args)
    elif args.impl == "reference" and args.workload in MESH_WORKLOADS:
        res = None if dist_env()[0] else {
            "impl": "reference",
            "unavailable": "the oracle field would need days per extraction at this size on the host; the "
                           "B200 line's cpu_baseline gives the oracle's marching time plus its sampled field cost"}
    elif args.impl == "reference":
        res = run_reference(args)
    elif args.workload in FIELD_WORKLOADS:
        res = run_field(args)
    elif args.workload in MESH_WORKLOADS:
        res = run_mesh(args)
    else:
        res = run_b200(args)
    if res is not None:
        print(json.dumps(res))


if __name__ == "__main__":
    main()
