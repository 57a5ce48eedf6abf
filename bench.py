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
DEFAULT_WORKLOAD = "surfaces1m_1080p"
# workloads rendered as a batch of views per GPU per step (the rest: one view)
VIEW_BATCHED = {"surfaces3m_views64": 8}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--mode", default="gof")
    ap.add_argument("--distortions", default="both")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the view-batched step and the opacity field timed after the headline")
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
# kernel: an ncu capture of one launch on the 100k-Gaussian 800x800 case (485.92 + 16.24
# MB, 43.28M contributing samples) scaled by the 1080p frame's contributing samples
# (291.08M): the backward's traffic is the per-sample L1 factors plus per-pixel state
# and the records its warps read.
MEASURED_TRAFFIC = {("surfaces1m_1080p", "gof", "both", "raster_backward"): round((485.92e6 + 16.24e6) * 291.08 / 43.28)}


def algorithmic_flops(mode, n_pairs_fwd):
    """Per-pair algorithmic FP32 flops of the raster forward: the sample equations of
    each mode (GOF: Q r, the ray peak, the offset, its quadratic form, the normal)."""
    per = {"radegs": 35, "gof": 70, "ambisur": 40}[mode]
    return per * n_pairs_fwd


POSES = 8  # orbit poses of the single-view workloads, cycled step by step


def linear_loss(images, ups):
    """sum over channels of <image, upstream>: one dot-product kernel per channel (and
    one scaling kernel per channel in the backward), the fixed seeded stand-in for a
    training loss whose adjoint of every image is its upstream tensor."""
    return sum(torch.vdot(images[ch].reshape(-1), ups[ch].reshape(-1)) for ch in CHANNELS)


def workload_label(args, n, width, height, views):
    return (f"{args.workload}: {n} Gaussians, {width}x{height}, mode {args.mode}, distortions {args.distortions}, "
            f"fwd+bwd, {views} view(s) per GPU per step")


class RenderJob:
    """The training step of a render workload on one rank: forward + backward of this
    rank's view(s) of the replicated scene against fixed seeded upstream gradients on
    every output channel, then (N > 1) one NCCL all-reduce of the [N,59] gradients.

    Pose schedule (the same at every N, so every N sees the same per-view costs):

    * single-view workloads: at step s every rank renders orbit pose s mod 8 (with
      ``distinct=True``, rank r renders pose (s + r) mod 8 instead, the load imbalance of
      a batch of different poses);
    * view-batched workloads: step s renders the 8N poses 8sN .. 8sN + 8N - 1 of the
      workload's 64 (mod 64), so one rank cycles through all 64 and eight ranks render
      all 64 every step.  During the warm-up rank r renders poses 8(r + sN) .. +7 and
      times each view; after it the ranks share the per-pose times (one all-reduce) and
      every timed step splits its 8N poses across the ranks by measured cost, longest
      first (distributed.balanced_views), so the close-up poses do not pile onto one rank.
    """

    def __init__(self, workload, dev, rank, world, mode, distortions):
        from splatforge_b200 import distributed, scenes
        from splatforge_b200.rasterizer import RasterSettings

        params, wl_cams = scenes.workload(workload, seed=0)
        self.per = VIEW_BATCHED.get(workload, 1)
        if self.per > 1:
            self.poses = wl_cams
        else:
            base = wl_cams[0]
            self.poses = scenes.orbit_cameras(POSES, base.width, base.height, 60.0 if "1080" in workload else 50.0,
                                              radius=3.0, seed=0)
        self.workload, self.rank, self.world, self.mode, self.distortions = workload, rank, world, mode, distortions
        self.settings = RasterSettings(mode=mode, distortions=distortions)
        self.H, self.W = self.poses[0].height, self.poses[0].width
        g = torch.Generator().manual_seed(1234 + rank)
        self.ups = {ch: torch.randn(self.H, self.W, 3 if ch in ("rgb", "normals") else 1, generator=g).to(dev)
                    for ch in CHANNELS}
        self.params = params
        self.p = params.to(dev).requires_grad_()
        self.n = self.p.means.shape[0]
        self.dev = dev
        self.reducer = distributed.GradientAllReduce(self.p.tensors(), timed=True)
        if world > 1:
            # the gradients accumulate in the all-reduce buffer itself (no copy in or out)
            self.reducer.bind()
        self.last = None
        self.costs = None      # per-pose render ms shared by all ranks (view-batched)
        self.view_events = []  # (pose, start, end) timed during the warm-up
        self.views_per_rank = None

    def pose_ids(self, s, distinct=False):
        if self.per == 1:
            return [((s + self.rank) if distinct else s) % len(self.poses)]
        if self.costs is None:
            base = self.per * (self.rank + s * self.world)
            return [(base + v) % len(self.poses) for v in range(self.per)]
        from splatforge_b200 import distributed

        step_poses = [(self.per * self.world * s + k) % len(self.poses) for k in range(self.per * self.world)]
        split = distributed.balanced_views(step_poses, self.costs, self.world)
        self.views_per_rank = [len(x) for x in split]
        return split[self.rank]

    def cams(self, s, distinct=False):
        return [self.poses[i] for i in self.pose_ids(s, distinct)]

    def step(self, s, distinct=False):
        from splatforge_b200 import rasterizer, scenes

        self.reducer.zero_grad()
        timing = self.per > 1 and self.costs is None
        out = None
        for i in self.pose_ids(s, distinct):
            if timing:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            view = scenes.activated(self.p)
            out = rasterizer.rasterize(view.means, view.quats, view.scales, view.opacities, view.sh, 3,
                                       self.poses[i], self.settings)
            loss = linear_loss(out, self.ups)
            loss.backward()
            if timing:
                ev[1].record()
                self.view_events.append((i, ev[0], ev[1]))
        self.reducer()
        self.last = out
        return out

    def share_costs(self):
        """After the warm-up (every rank): the per-pose render times become one table."""
        from splatforge_b200 import distributed

        if self.per == 1 or self.costs is not None or not self.view_events:
            return  # (the same on every rank: all ran the same warm-up steps)
        torch.cuda.synchronize()
        local = {}
        for i, a, b in self.view_events:
            local[i] = max(local.get(i, 0.0), a.elapsed_time(b))
        self.view_events = []
        self.costs = distributed.shared_view_costs(local, len(self.poses), device=self.dev)

    def pixels_per_step(self):
        return self.H * self.W * self.per * self.world


def _max_over_ranks(value, dev, world):
    import torch.distributed as dist

    t = torch.tensor([float(value)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gather(values, dev, world):
    """Every rank's list of floats, on every rank (rank order)."""
    import torch.distributed as dist

    t = torch.tensor([float(v) for v in values], device=dev)
    if world == 1:
        return [t.tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def time_steps(job, steps, warmup, distinct=False):
    """Warm-up steps, then ``steps`` steps bracketed by a barrier and a synchronize on
    both sides and timed with CUDA events on the launching stream.  Returns (mean ms
    per step of this rank, per-step ms of this rank)."""
    import torch.distributed as dist

    for s in range(warmup):
        job.step(s, distinct)
    job.share_costs()
    torch.cuda.synchronize()
    job.reducer.events.clear()
    if job.world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    from splatforge_b200 import rasterizer

    import gc

    stats0 = torch.cuda.memory_stats()
    reruns0 = rasterizer.COUNTERS["l1_reruns"]
    rebins0 = rasterizer.COUNTERS["bin_reruns"]
    host = []
    gc_ms = [0.0]
    gc_t = [0.0]

    def gc_cb(phase, info):
        if phase == "start":
            gc_t[0] = time.perf_counter()
        else:
            gc_ms[0] += 1e3 * (time.perf_counter() - gc_t[0])

    gc.callbacks.append(gc_cb)
    ev[0].record()
    for s in range(steps):
        h0 = time.perf_counter()
        job.step(s, distinct)
        ev[s + 1].record()
        host.append(1e3 * (time.perf_counter() - h0))
    torch.cuda.synchronize()
    gc.callbacks.remove(gc_cb)
    if job.world > 1:
        dist.barrier()
    stats1 = torch.cuda.memory_stats()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    # host-side launch time per step and the allocator's device allocations in the timed
    # steps (a step whose device time exceeds its peers' with host time to match was held
    # up on the host)
    job.diag = {"host_ms": [round(x, 2) for x in host],
                "device_allocs": stats1.get("num_device_alloc", 0) - stats0.get("num_device_alloc", 0),
                "alloc_retries": stats1.get("num_alloc_retries", 0) - stats0.get("num_alloc_retries", 0),
                "device_frees": stats1.get("num_device_free", 0) - stats0.get("num_device_free", 0),
                "l1_reruns": rasterizer.COUNTERS["l1_reruns"] - reruns0,
                "bin_reruns": rasterizer.COUNTERS["bin_reruns"] - rebins0, "gc_ms": round(gc_ms[0], 2)}
    return ev[0].elapsed_time(ev[-1]) / steps, per


def _median(xs):
    xs = sorted(xs)
    return xs[len(xs) // 2] if xs else None


def run_b200(args):
    import torch.distributed as dist

    from splatforge_b200 import distributed, rasterizer, scenes
    from splatforge_b200.renderer import B200Renderer

    rank, world, local = distributed.init_from_env(backend="nccl", timeout_s=300)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    job = RenderJob(args.workload, dev, rank, world, args.mode, args.distortions)
    n, H, W = job.n, job.H, job.W

    # warm-up (also settles the per-image-size L1 capacity), then the timed steps with
    # per-kernel events around the dominant kernels
    for s in range(args.warmup):
        job.step(s)
    torch.cuda.synchronize()
    n_isect = job.last["n_isect"]
    prof = {"fwd": [], "bwd": []}
    rasterizer.PROFILE = prof
    launches0 = rasterizer.kernel_launches()
    clocks = ClockSampler(local).start() if rank == 0 else None
    ms_rank, per_step = time_steps(job, args.steps, 0)
    rasterizer.PROFILE = None
    launches = rasterizer.kernel_launches() - launches0
    clk = clocks.stop() if clocks else None
    ms = _max_over_ranks(ms_rank, dev, world)
    pixels = job.pixels_per_step()
    value = pixels / (ms * 1e-3) / 1e6
    fwd_times = [a.elapsed_time(b) for a, b in prof["fwd"]]
    bwd_times = [a.elapsed_time(b) for a, b in prof["bwd"]]
    # per forward launch: (pairs evaluated, pairs contributing); one backward per forward
    launch_pairs = [tuple(int(v) for v in c.tolist()) for c in prof.get("counters", [])]
    counters = [sum(c[i] for c in launch_pairs) // max(len(launch_pairs), 1) for i in (0, 1)]
    coll = job.reducer.timings_ms() or (0.0, 0.0, 0.0)
    ranks = _gather([_median(per_step), *coll, _median(fwd_times) or 0.0, _median(bwd_times) or 0.0], dev, world)

    distinct = None
    if world > 1 and job.per == 1:
        # the same step with a different pose on every rank: the max over ranks then also
        # carries the spread of per-pose cost
        dms, _ = time_steps(job, args.steps, 2, distinct=True)
        dms = _max_over_ranks(dms, dev, world)
        distinct = {"ms_per_step": round(dms, 3), "value": round(pixels / (dms * 1e-3) / 1e6, 3),
                    "poses": "rank r renders orbit pose (s + r) mod 8 at step s"}

    e2e = None if args.no_e2e else e2e_render(job, args, dev, rank, world, B200Renderer, distributed, scenes)

    result = None
    if rank == 0:
        fwd, bwd = _median(fwd_times), _median(bwd_times)
        peaks = measured_peaks()
        sm_mhz = (clk or {}).get("sm_mhz") or 1965.0
        fp32_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
        roof = None
        if bwd is not None and len(launch_pairs) == len(bwd_times) == len(fwd_times):
            # algorithmic flops of every launch over the launches' summed event time
            dom, times = ("raster_backward", bwd_times) if bwd >= (fwd or 0) else ("raster_forward", fwd_times)
            dom_ms = sum(times) / len(times)
            flops = sum(algorithmic_flops(args.mode, c[0]) for c in launch_pairs) * (2 if dom == "raster_backward" else 1)
            achieved = flops / (sum(times) * 1e-3) / 1e12
            roof = {"bound": "fp32", "kernel": dom, "achieved": round(achieved, 3),
                    "peak": round(fp32_peak, 2), "unit": "TFLOP/s", "frac": round(achieved / fp32_peak, 4),
                    "traffic": MEASURED_TRAFFIC.get((args.workload, args.mode, args.distortions, dom)),
                    "traffic_unit": "bytes per launch", "kernel_ms": round(dom_ms, 4),
                    "peak_source": f"FP32 SIMT 148 SM x 128 lanes x 2 at the sampled {sm_mhz:.0f} MHz",
                    "hbm_peak_gbs": peaks.get("hbm_gbs")}
        poses = ("every rank renders orbit pose s mod 8 at step s" if job.per == 1 else
                 f"step s renders poses 8sN .. 8sN + 8N - 1 of the {len(job.poses)} (mod {len(job.poses)}), split "
                 "across the ranks by the per-pose render times measured in the warm-up (longest first)")
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": "Mpix/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded surface-sampled scene, seeded orbit camera poses)",
            "config": {"workload": workload_label(args, n, W, H, job.per),
                       "parallelism": f"view-sharded dp{world}, NCCL all-reduce of [N,59] grads" if world > 1 else "single GPU",
                       "poses": poses, "views_per_s": round(world * job.per / (ms * 1e-3), 3),
                       "n_isect": int(n_isect),
                       "l2_policy": "inputs larger than L2 (236 MB parameters + records per step)",
                       "fwd_ms": fwd, "bwd_ms": bwd, "pairs_evaluated": counters[0],
                       "pairs_contributing": counters[1], "pairs_in_tile_lists": int(n_isect) * 256},
            "ranks": {"step_ms_median": [round(r[0], 3) for r in ranks],
                      "pack_ms": [round(r[1], 3) for r in ranks], "allreduce_ms": [round(r[2], 3) for r in ranks],
                      "unpack_ms": [round(r[3], 3) for r in ranks],
                      "raster_fwd_ms": [round(r[4], 3) for r in ranks], "raster_bwd_ms": [round(r[5], 3) for r in ranks],
                      "collective_share": round(_median([(r[1] + r[2] + r[3]) / r[0] for r in ranks if r[0]]) or 0.0, 4)},
            "distinct_poses": distinct,
            "steps_this_rank": {"step_ms": [round(x, 2) for x in per_step], **job.diag},
            "gpu_launches": int(launches),
            "clocks": clk, "e2e": e2e, "roofline": roof,
        }
        # the CPU baseline is timed once, at N=1 (other ranks would compete for the cores)
        result["cpu_baseline"] = cpu_baseline(args) if world == 1 and not args.no_cpu_baseline else None
    del job
    torch.cuda.empty_cache()
    if not args.no_secondary and args.workload == DEFAULT_WORKLOAD:
        sec = secondary(args, dev, rank, world)
        if rank == 0:
            result["secondary"] = sec
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def e2e_render(job, args, dev, rank, world, B200Renderer, distributed, scenes):
    """End to end through the public renderer API (``B200Renderer.render``): pinned host
    parameters in, loss out.  Every step uploads its parameters; the upload of step k+1
    runs on a copy stream into the second of two parameter buffers while step k renders
    (a prefetching loader), and every upload lies inside the timed region."""
    import torch.distributed as dist

    renderer = B200Renderer(settings_config(job.settings), mode=args.mode)
    host = [t.detach().cpu().pin_memory() for t in job.params.tensors()]
    bufs = [[torch.empty_like(t, device=dev) for t in host] for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    loss_host = torch.empty((), pin_memory=True)
    reducers = [distributed.GradientAllReduce(b) for b in bufs]
    if world > 1:
        for r in reducers:
            r.bind()
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
            reducers[slot].zero_grad()
            sp = scenes.SceneParams(*dev_params, sh_degree=3)
            total = 0.0
            for c in job.cams(k):
                v = scenes.activated(sp)
                o = renderer.render(v, c, distortions=args.distortions)
                loss = linear_loss({ch: getattr(o, ch) for ch in CHANNELS}, job.ups)
                loss.backward()
                total = total + loss.detach()
            reducers[slot]()
            loss_host.copy_(total, non_blocking=True)
            for d in dev_params:
                d.requires_grad_(False)
            freed[slot].record()

    e2e_steps(max(3, args.warmup), None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    e2e_steps(args.steps, a0)
    a1.record()
    torch.cuda.synchronize()
    ems = _max_over_ranks(a0.elapsed_time(a1) / args.steps, dev, world)
    return {"value": round(job.pixels_per_step() / (ems * 1e-3) / 1e6, 3), "unit": "Mpix/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "ms_per_step": round(ems, 3),
            "upload": "pinned host -> device every step, overlapped with the previous step's render"}


def secondary(args, dev, rank, world):
    """The view-batched training step and the opacity field, timed in the same run
    (values over all ranks; time = max over ranks)."""
    out = {}
    job = RenderJob("surfaces3m_views64", dev, rank, world, "gof", "l1")
    # warm-up over every pose a rank renders (64 / (8 N) steps), so that the per-size L1
    # sample capacity has settled before the timed steps
    warm = max(3, len(job.poses) // (job.per * world))
    ms_rank, per_step = time_steps(job, max(3, min(args.steps, 10)), warm)
    ms = _max_over_ranks(ms_rank, dev, world)
    coll = job.reducer.timings_ms() or (0.0, 0.0, 0.0)
    ranks = _gather([_median(per_step), *coll], dev, world)
    views = world * job.per
    out["view_batched"] = {
        "metric": "views/s", "value": round(views / (ms * 1e-3), 3), "unit": "views/s",
        "mpix_per_s": round(job.pixels_per_step() / (ms * 1e-3) / 1e6, 3), "ms_per_step": round(ms, 3),
        "workload": f"surfaces3m_views64: {job.n} Gaussians, {job.W}x{job.H}, mode gof, distortions l1 "
                    f"(the training profile), fwd+bwd, {job.per} views per GPU per step, {views} per step",
        "poses": f"step s renders poses 8sN .. 8sN + 8N - 1 of the {len(job.poses)} (mod {len(job.poses)}), "
                 "split across the ranks by the per-pose render times measured in the warm-up (longest first)",
        "views_per_rank_last_step": job.views_per_rank,
        "warmup_steps": warm, "step_ms_this_rank": [round(x, 2) for x in per_step], "diag_this_rank": job.diag,
        "value_median_step": round(views / (_median(per_step) * 1e-3), 3),
        "step_ms_median": [round(r[0], 3) for r in ranks], "allreduce_ms": [round(r[2], 3) for r in ranks],
        "pack_unpack_ms": [round(r[1] + r[3], 3) for r in ranks]}
    del job
    torch.cuda.empty_cache()
    # the C3 frame in the other two modes (the headline is GOF), every output channel
    for mode in ("radegs", "ambisur"):
        job = RenderJob(DEFAULT_WORKLOAD, dev, rank, world, mode, "both")
        ms_rank, per_step = time_steps(job, POSES, 3)
        ms = _max_over_ranks(ms_rank, dev, world)
        out[f"c3_{mode}"] = {
            "metric": "fwd+bwd rendered Mpix/s", "unit": "Mpix/s",
            "value": round(job.pixels_per_step() / (ms * 1e-3) / 1e6, 3), "ms_per_step": round(ms, 3),
            "workload": workload_label(argparse.Namespace(workload=DEFAULT_WORKLOAD, mode=mode, distortions="both"),
                                       job.n, job.W, job.H, 1),
            "steps": POSES, "warmup": 3, "n_isect_last": int(job.last["n_isect"])}
        del job
        torch.cuda.empty_cache()
    field = field_measure(dev, rank, world, steps=2, warmup=1, e2e=False)
    out["opacity_field"] = field
    torch.cuda.empty_cache()
    return out


FIELD_WORKLOADS = {"field2m_views32"}
FIELD_SHARDS = 8  # the query set is cut into 8 shards; rank r evaluates shard r
# FP32 flops of one evaluated (query, candidate) pair of the culled field (multiplies
# and adds, an FMA as two, plus one exp): origin - mean 3, Q d 15, d.Qd 5, the peak
# (dot, divide) 6, the offset at min(peak, distance) 6, its quadratic form 20, the
# response 2, the transmittance update 2
FIELD_FLOP_PER_PAIR = 59


def field_measure(dev, rank, world, *, steps, warmup, e2e=True, no_cpu_baseline=True, workload="field2m_views32"):
    """GOF opacity field over an extraction grid (9 points per Gaussian + 2M uniform),
    2M Gaussians, 32 view origins; rank r evaluates shard r mod 8 of the ~20M queries
    (weak scaling: 8 shards at 8 GPUs), with no collective on the data path.  Returns the
    rank-0 record (None elsewhere)."""
    from splatforge_b200 import distributed, ops, rasterizer, scenes

    params, cams = scenes.workload(workload, seed=0)
    view = scenes.activated(params)
    queries = scenes.field_queries(params, 2_000_000, seed=0)
    q = queries.shape[0]
    lo, hi = distributed.query_shard(q, rank, FIELD_SHARDS)
    host = {"pts": queries[lo:hi].contiguous().pin_memory(), "means": view.means.contiguous().pin_memory(),
            "Q": scenes.inverse_covariances(params).contiguous().pin_memory(),
            "opac": view.opacities.contiguous().pin_memory(),
            "origins": torch.stack([c.origin for c in cams]).contiguous().pin_memory()}
    d = {k: v.to(dev) for k, v in host.items()}
    n_q = hi - lo
    state = {"stats": None, "out": None}

    def step():
        state["out"] = ops.opacity_field_culled(d["pts"], d["means"], d["Q"], d["opac"], d["origins"],
                                                stats=state["stats"])
        return state["out"]

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    launches0 = rasterizer.kernel_launches()
    state["stats"] = {}
    clocks = ClockSampler(torch.cuda.current_device()).start() if rank == 0 else None
    ms_rank, _ = _timed(step, steps, world)
    clk = clocks.stop() if clocks else None
    launches = rasterizer.kernel_launches() - launches0
    stats, out = state["stats"], state["out"]
    state["stats"] = None
    ms = _max_over_ranks(ms_rank, dev, world)
    value = n_q * world / (ms * 1e-3)
    pairs = stats.get("pairs_evaluated")
    query_ms = stats.get("query_ms")

    e2e_rec = None
    if e2e:
        # queries and scene from pinned host memory in, field values out
        field_host = torch.empty((n_q,), pin_memory=True)
        h2d = sum(v.numel() * v.element_size() for v in host.values())

        def e2e_step():
            for k, v in host.items():
                d[k].copy_(v, non_blocking=True)
            field_host.copy_(step(), non_blocking=True)

        ems, _ = _timed(e2e_step, steps, world)
        ems = _max_over_ranks(ems, dev, world)
        e2e_rec = {"value": round(n_q * world / (ems * 1e-3), 1), "unit": "queries/s",
                   "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(n_q * 4), "ms_per_step": round(ems, 3)}
    if rank != 0:
        return None
    roof = None
    if pairs and query_ms:
        sm_mhz = (clk or {}).get("sm_mhz") or 1965.0
        peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
        achieved = FIELD_FLOP_PER_PAIR * pairs / (query_ms * 1e-3) / 1e12
        roof = {"bound": "fp32", "kernel": "cfield_query", "achieved": round(achieved, 3), "peak": round(peak, 2),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                "kernel_ms": round(query_ms, 3), "pairs_evaluated": int(pairs),
                "flop_per_pair": FIELD_FLOP_PER_PAIR,
                "peak_source": f"FP32 SIMT 148 SM x 128 lanes x 2 at the sampled {sm_mhz:.0f} MHz"}
    return {
        "metric": "GOF opacity-field queries/s (2M Gaussians, 32 views)", "value": round(value, 1),
        "unit": "queries/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded surface-sampled scene, exporter-shaped query grid)",
        "config": {"workload": f"{workload}: {params.means.shape[0]} Gaussians, {len(cams)} origins, "
                               f"{n_q} queries per GPU ({q} in {FIELD_SHARDS} shards)",
                   "parallelism": f"query-sharded x{world}, no collective" if world > 1 else "single GPU",
                   "path": "culled per-view cube-map candidate lists (contributions <= 1e-7 dropped)",
                   "field_mean": round(float(out.mean().item()), 6) if out is not None else None},
        "gpu_launches": int(launches), "clocks": clk, "e2e": e2e_rec, "roofline": roof,
        "cpu_baseline": None if no_cpu_baseline else field_cpu_baseline(host),
    }


def _timed(fn, steps, world):
    """``steps`` calls of ``fn`` between a barrier and a synchronize on both sides, timed
    with CUDA events on the current stream; (mean ms per call, per-call ms)."""
    import torch.distributed as dist

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record()
    for s in range(steps):
        fn()
        ev[s + 1].record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return ev[0].elapsed_time(ev[-1]) / steps, [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]


def run_field(args):
    import torch.distributed as dist

    from splatforge_b200 import distributed

    rank, world, local = distributed.init_from_env(backend="nccl", timeout_s=300)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    result = field_measure(dev, rank, world, steps=args.steps, warmup=args.warmup, e2e=not args.no_e2e,
                           no_cpu_baseline=args.no_cpu_baseline or world > 1, workload=args.workload)
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


REF_INSTALL = ROOT / "baseline" / "_ref"


def reference_importable():
    """True when the reference package is installed in baseline/_ref (pip --target) and
    imports; its renderer is then the CPU baseline instead of the oracle port."""
    if not (REF_INSTALL / "splatforge").is_dir():
        return False
    if str(REF_INSTALL) not in sys.path:
        sys.path.append(str(REF_INSTALL))
    try:
        import splatforge.studio.batched_renderer  # noqa: F401
    except Exception:
        return False
    return True


def _full_frame_lists(view, cam, mode):
    """The frame's exact tile lists (the oracle's projection and binning, which equal the
    reference's tile_members bit for bit) and per-tile pixel counts."""
    import numpy as np

    from oracle import binning as oracle_binning
    from oracle import render as oracle_render

    with torch.no_grad():
        m, _, _, xy, _, filt = oracle_render.project(view, cam, 0.3, 0.01)
        _, radii = oracle_render.conic_and_radius(filt, 2.0 if mode == "ambisur" else 3.0)
    bounds = torch.cat((xy, radii[:, None], m[:, 2:3]), 1).numpy()
    offsets, ids, _ = oracle_binning.tile_lists(bounds, width=cam.width, height=cam.height, tile_size=16,
                                                near=0.01, far=1e4)
    cols, rows = (cam.width + 15) // 16, (cam.height + 15) // 16
    t = np.arange(rows * cols)
    pix = np.minimum(16, cam.height - (t // cols) * 16) * np.minimum(16, cam.width - (t % cols) * 16)
    return bounds, offsets, ids, pix, cols, rows


class RefCropSampler:
    """The reference's own renderer (``BatchedTorchRenderer`` from baseline/_ref, eager,
    on the host cores) on the bench's first pose, extrapolated to the full frame:

    * fixed cost: one render + backward of a window that no Gaussian reaches, with the
      whole scene (projection, conics, colours, mode extras, the tile-binning loop over
      every Gaussian), timed once; plus the binning appends of the full frame
      (``tile_members`` on a 1/16 sample of the Gaussians over the full frame, x16);
    * tile work: each sample renders + back-propagates one random 32x32 window (2x2
      tiles) through the reference's public ``render`` with only the Gaussians that
      reach the window (their tile lists, and so the reference's padded batches, are
      the full frame's); the sampled seconds (less the subset's share of the fixed
      cost) per unit of work (list length x tile pixels) times the frame's work.
    """

    kind = "reference"

    def __init__(self, args, threads, window=2):
        import numpy as np

        from splatforge.studio.batched_renderer import BatchedTorchRenderer
        from splatforge.studio.cameras import Camera
        from splatforge.studio.config import RenderConfig
        from splatforge.studio.renderers import GaussianView
        from splatforge.studio.tile_binning import tile_members

        from splatforge_b200 import scenes

        torch.set_num_threads(threads)
        self.threads, self.window = threads, window
        self.GaussianView, self.Camera = GaussianView, Camera
        self.distortions = args.distortions
        params, cams = scenes.workload(args.workload, seed=0)
        self.cam = cams[0]
        self.params = params
        self.n = params.means.shape[0]
        self.renderer = BatchedTorchRenderer(RenderConfig(), mode=args.mode)
        view = scenes.activated(params)
        bounds, self.offsets, self.ids, self.pix, self.cols, self.rows = _full_frame_lists(view, self.cam, args.mode)
        lens = np.diff(self.offsets)
        self.tile_work = lens * self.pix
        self.frame_work = float(self.tile_work.sum())
        # the fixed cost: a window left of the image that no Gaussian reaches
        t0 = time.perf_counter()
        self._render(np.arange(self.n), -100000, -100000)
        self.t_fixed = time.perf_counter() - t0
        rng = np.random.default_rng(11)
        sub = np.sort(rng.choice(self.n, self.n // 16, replace=False))
        t0 = time.perf_counter()
        tile_members(bounds[sub], width=self.cam.width, height=self.cam.height, tile_size=16, near=0.01, far=1e4)
        self.t_bin = 16 * (time.perf_counter() - t0)
        # windows of full tiles with any work
        wins = []
        for ty in range(0, self.rows - window + 1):
            if (ty + window) * 16 > self.cam.height:
                continue
            for tx in range(0, self.cols - window + 1):
                if (tx + window) * 16 > self.cam.width:
                    continue
                tiles = [(ty + a) * self.cols + tx + b for a in range(window) for b in range(window)]
                w = float(self.tile_work[tiles].sum())
                if w > 0:
                    wins.append((tx, ty, tiles, w))
        self.windows = wins
        self.samples = []  # (seconds, fixed-cost share, work)
        self.setup_seconds = None

    def _render(self, subset, left, top):
        from splatforge_b200 import scenes

        idx = torch.as_tensor(subset, dtype=torch.int64)
        p = scenes.SceneParams(*(t[idx].clone() for t in self.params.tensors()), sh_degree=3).requires_grad_()
        v = scenes.activated(p)
        gv = self.GaussianView(means=v.means, quats=v.quats, scales=v.scales, opacities=v.opacities, sh=v.sh,
                               sh_degree=3)
        size = 16 * self.window
        crop = self.cam.crop(left, top, size, size)
        cam = self.Camera(K=crop.K, world_to_camera=crop.world_to_camera, width=size, height=size)
        out = self.renderer.render(gv, cam, distortions=self.distortions)
        loss = sum(getattr(out, ch).sum() for ch in CHANNELS)
        loss.backward()

    def sample(self, rng):
        import numpy as np

        tx, ty, tiles, work = self.windows[int(rng.integers(len(self.windows)))]
        subset = np.unique(np.concatenate([self.ids[self.offsets[t]:self.offsets[t + 1]] for t in tiles]))
        t0 = time.perf_counter()
        self._render(subset, 16 * tx, 16 * ty)
        dt = time.perf_counter() - t0
        self.samples.append((dt, self.t_fixed * len(subset) / self.n, work))
        return dt

    def frame_seconds(self):
        spent = sum(max(dt - share, 0.0) for dt, share, _ in self.samples)
        work = sum(w for _, _, w in self.samples)
        return self.t_fixed + self.t_bin + spent / work * self.frame_work

    def describe(self):
        spent = sum(dt for dt, _, _ in self.samples)
        return (f"the reference's BatchedTorchRenderer (baseline/_ref, eager, {self.threads} threads) fwd+bwd of "
                f"{len(self.samples)} random {16 * self.window}x{16 * self.window} windows of the "
                f"{self.cam.width}x{self.cam.height} view with the Gaussians reaching them ({spent:.1f} s), "
                f"extrapolated by tile work (list length x pixels) to the frame; plus its fixed per-frame cost with "
                f"all {self.n} Gaussians ({self.t_fixed:.1f} s, timed once) and the frame's binning appends "
                f"({self.t_bin:.1f} s, from a 1/16 sample)")


class PortSampler:
    """The oracle port (CPU restatement of the reference's renderer) on the same view,
    used when the reference is not installed: the full-scene projection and binning and
    its backward, timed once, plus uniformly sampled padded tile batches (formed as the
    Torch provider forms them) times the batch count."""

    kind = "port"

    def __init__(self, args, threads):
        from oracle import render as oracle_render
        from splatforge_b200 import scenes

        torch.set_num_threads(threads)
        self.threads = threads
        self.render = oracle_render
        params, cams = scenes.workload(args.workload, seed=0)
        self.cam = cams[0]
        self.n = params.means.shape[0]
        self.leaves = params.detach_clone().requires_grad_()
        t0 = time.perf_counter()
        view = scenes.activated(self.leaves)
        self.ctx = oracle_render.prepare(view, self.cam, mode=args.mode, distortions=args.distortions)
        self.t_prep = time.perf_counter() - t0
        names = ("xy", "conic", "colors", "ray_colors", "opacity", "m", "normals", "gain", "qinv", "plane")
        inter = [self.ctx[k] for k in names if self.ctx[k].requires_grad]
        g = torch.Generator().manual_seed(7)
        ups = [torch.randn(t.shape, generator=g) for t in inter]
        t0 = time.perf_counter()
        torch.autograd.grad(inter, self.leaves.tensors(), grad_outputs=ups, retain_graph=True, allow_unused=True)
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
        self.samples = []
        self.setup_seconds = None

    def sample(self, rng):
        tiles, longest = self.batches[int(rng.integers(len(self.batches)))]
        c0 = time.perf_counter()
        out = self.render.render_batch(self.ctx, tiles, longest)
        loss = (out * self.up[: out.shape[1]]).sum()
        if loss.requires_grad:
            torch.autograd.grad(loss, self.inter, allow_unused=True)
        dt = time.perf_counter() - c0
        self.samples.append(dt)
        return dt

    def frame_seconds(self):
        return self.t_prep + len(self.batches) * (sum(self.samples) / len(self.samples)) + self.t_prep_bwd

    def describe(self):
        return (f"oracle port fwd+bwd of {len(self.samples)} uniformly sampled tile batches (of {len(self.batches)}, "
                f"formed as the Torch provider forms them) of the {self.cam.width}x{self.cam.height} view "
                f"({sum(self.samples):.1f} s), plus the full-scene projection/binning ({self.t_prep:.1f} s) and "
                f"its backward ({self.t_prep_bwd:.1f} s), timed once")


def cpu_sampler(args, threads):
    t0 = time.perf_counter()
    sampler = RefCropSampler(args, threads) if reference_importable() else PortSampler(args, threads)
    sampler.setup_seconds = time.perf_counter() - t0
    return sampler


def cpu_baseline(args, budget_s=10.0):
    """The CPU figure beside the B200 line (N = 1): the reference's renderer (or the port)
    on all host cores, sampled for about ``budget_s`` seconds after its set-up."""
    import numpy as np

    threads = os.cpu_count() or 1
    try:
        sampler = cpu_sampler(args, threads)
        rng = np.random.default_rng(0)
        spent = 0.0
        while spent < budget_s or not sampler.samples:
            spent += sampler.sample(rng)
        frame = sampler.frame_seconds()
    except Exception as exc:  # the baseline must not hide the GPU result
        return {"value": None, "unit": "Mpix/s", "cores": threads, "kind": "reference", "sample": f"failed: {exc}"}
    return {"value": round(sampler.cam.width * sampler.cam.height / frame / 1e6, 6), "unit": "Mpix/s",
            "cores": threads, "kind": sampler.kind, "extrapolated": True, "frame_seconds": round(frame, 1),
            "sample": sampler.describe()}


def run_reference(args):
    """The reference arm: the reference's renderer (or the port) on the host cores; each
    step is one bounded sample (a window of tiles, or a tile batch for the port), and
    ``value`` is the full frame's Mpix/s extrapolated from all samples.  ``ms_per_step``
    is the measured wall time of a step."""
    import numpy as np

    rank, world, _ = dist_env()
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    sampler = cpu_sampler(args, threads)
    rng = np.random.default_rng(0)
    for _ in range(args.warmup):
        sampler.sample(rng)
    sampler.samples.clear()
    step_s = [sampler.sample(rng) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    frame = sampler.frame_seconds()
    value = sampler.cam.width * sampler.cam.height / frame / 1e6
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "Mpix/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sum(step_s) / len(step_s), 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded surface-sampled scene, seeded orbit camera poses)",
        "extrapolated": True,
        "config": {"workload": workload_label(args, sampler.n, sampler.cam.width, sampler.cam.height, 1),
                   "frame_seconds_extrapolated": round(frame, 1), "samples": len(step_s),
                   "setup_seconds": round(sampler.setup_seconds, 1), "wall_seconds": round(wall, 1)},
        "cpu_baseline": {"value": round(value, 6), "unit": "Mpix/s", "cores": threads, "kind": sampler.kind,
                         "extrapolated": True, "sample": sampler.describe()},
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
