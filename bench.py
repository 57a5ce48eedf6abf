"""Forward + backward throughput of the B200 rasterizer (Mpix/s), 1..8 GPUs.

Workload (default): the 1M-Gaussian surface scene at 1920x1080, 60 deg FOV,
GOF mode with the full distortion set ("both": RGB, expected depth, median depth,
normal, L1 and L2 distortion, ray colour, ambiguity) forward + backward against
fixed seeded upstream gradients on every output.  Each rank renders its own view
of the replicated scene per step; with N > 1 ranks the per-Gaussian gradients
(59 floats per Gaussian) are all-reduced with NCCL every step (view-sharded data
parallelism).  ``value`` = all ranks' rendered pixels / max-over-ranks step time.

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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", default="surfaces1m_1080p")
    ap.add_argument("--mode", default="gof")
    ap.add_argument("--distortions", default="both")
    ap.add_argument("--no-e2e", action="store_true")
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


def algorithmic_flops(mode, n_pairs_fwd):
    """Per-pair algorithmic FP32 flops of the raster forward (SURVEY/DESIGN table)."""
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
    params, _ = scenes.workload(args.workload, seed=0)
    base_cam = scenes.workload(args.workload, seed=0)[1][0]
    cams = scenes.orbit_cameras(max(8, world), base_cam.width, base_cam.height, 60.0 if "1080" in args.workload else 50.0,
                                radius=3.0, seed=0)
    cam = cams[0] if world == 1 else cams[rank]
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
        view = scenes.activated(p)
        out = rasterizer.rasterize(view.means, view.quats, view.scales, view.opacities, view.sh, 3, cam, settings)
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
    pixels = H * W * world
    value = pixels / (ms * 1e-3) / 1e6

    # end to end through the public renderer API: pinned host parameters in, loss out
    e2e = None
    if not args.no_e2e:
        renderer = B200Renderer(settings_config(settings), mode=args.mode)
        host = [t.detach().cpu().pin_memory() for t in params.tensors()]
        dev_params = [torch.empty_like(t, device=dev) for t in host]
        h2d = sum(t.numel() * t.element_size() for t in host)
        loss_host = torch.empty((), pin_memory=True)
        e2e_reducer = distributed.GradientAllReduce(dev_params)

        def e2e_step():
            for d, h in zip(dev_params, host):
                d.copy_(h, non_blocking=True)
            for d in dev_params:
                d.requires_grad_(True)
                d.grad = None
            sp = scenes.SceneParams(*dev_params, sh_degree=3)
            v = scenes.activated(sp)
            o = renderer.render(v, cam, distortions=args.distortions)
            loss = sum((getattr(o, ch) * ups[ch]).sum() for ch in CHANNELS)
            loss.backward()
            e2e_reducer()
            loss_host.copy_(loss.detach(), non_blocking=True)
            for d in dev_params:
                d.requires_grad_(False)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(args.steps):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        ems = a0.elapsed_time(a1) / args.steps
        te = torch.tensor([ems], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        ems = float(te.item())
        e2e = {"value": round(pixels / (ems * 1e-3) / 1e6, 3), "unit": "Mpix/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "ms_per_step": round(ems, 3)}

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
                    "traffic": None, "kernel_ms": round(dom_ms, 4),
                    "peak_source": f"FP32 SIMT 148 SM x 128 lanes x 2 at the sampled {sm_mhz:.0f} MHz",
                    "hbm_peak_gbs": peaks.get("hbm_gbs")}
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": "Mpix/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded surface-sampled scene, random camera poses)",
            "config": {"workload": f"{args.workload}: {n} Gaussians, {W}x{H}, mode {args.mode}, "
                                   f"distortions {args.distortions}, fwd+bwd, 1 view per GPU per step",
                       "parallelism": f"view-sharded dp{world}, NCCL all-reduce of [N,59] grads" if world > 1 else "single GPU",
                       "views_per_s": round(world / (ms * 1e-3), 3), "n_isect": int(n_isect),
                       "l2_policy": "inputs larger than L2 (236 MB parameters + records per step)",
                       "fwd_ms": fwd, "bwd_ms": bwd, "pairs_evaluated": counters[0],
                       "pairs_contributing": counters[1], "pairs_in_tile_lists": int(n_isect) * 256},
            "gpu_launches": int(launches),
            "clocks": clk, "e2e": e2e, "roofline": roof,
        }
        result["cpu_baseline"] = cpu_baseline(args)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


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


def cpu_crop_sample(args, threads, budget_s=20.0):
    """The oracle (CPU port of the Torch provider) on tile-aligned crops of the same
    view; throughput extrapolated to the full frame by tile-list work."""
    import numpy as np

    from oracle import binning
    from oracle import render as oracle_render
    from splatforge_b200 import scenes

    torch.set_num_threads(threads)
    params, cams = scenes.workload(args.workload, seed=0)
    cam = cams[0]
    view = scenes.activated(params)
    t0 = time.perf_counter()
    m, _, _, xy, _, filt = oracle_render.project(view, cam, 0.3, 0.01)
    _, radii = oracle_render.conic_and_radius(filt, 3.0)
    bounds = torch.cat((xy, radii[:, None], m[:, 2:3]), 1).numpy()
    offsets, _, _ = binning.tile_lists(bounds, width=cam.width, height=cam.height, tile_size=16, near=0.01, far=1e4)
    t_setup = time.perf_counter() - t0
    tiles_x = (cam.width + 15) // 16
    lens = np.diff(offsets)
    work_full = float((lens * 256).sum())
    # crops of 2x2 tiles around the busiest part of the image until the budget is used
    order = np.argsort(-lens)
    done_work, t_crop, pix = 0.0, 0.0, 0
    for t in order[:: max(1, len(order) // 64)]:
        tx, ty = int(t % tiles_x), int(t // tiles_x)
        crop = cam.crop(tx * 16, ty * 16, 16, 16)
        p = params.detach_clone().requires_grad_()
        v = scenes.activated(p)
        c0 = time.perf_counter()
        out = oracle_render.render(v, crop, mode=args.mode, distortions=args.distortions)
        loss = sum(out[ch].sum() for ch in CHANNELS)
        loss.backward()
        t_crop += time.perf_counter() - c0
        done_work += float(lens[t] * 256)
        pix += 256
        if t_crop > budget_s:
            break
    # each crop re-projects the whole scene: remove that share using the setup timing
    per_tile_overhead = t_setup
    t_tiles = max(t_crop - per_tile_overhead * (pix // 256), t_crop * 0.05)
    t_full = t_setup + t_tiles * (work_full / max(done_work, 1.0))
    mpix = cam.width * cam.height / t_full / 1e6
    return mpix, {"tiles": pix // 256, "crop_seconds": round(t_crop, 2), "setup_seconds": round(t_setup, 2),
                  "extrapolated_full_frame_seconds": round(t_full, 1)}


def cpu_baseline(args):
    threads = os.cpu_count() or 1
    try:
        mpix, info = cpu_crop_sample(args, threads)
    except Exception as exc:  # the baseline must not hide the GPU result
        return {"value": None, "unit": "Mpix/s", "cores": threads, "kind": "port", "sample": f"failed: {exc}"}
    return {"value": round(mpix, 6), "unit": "Mpix/s", "cores": threads, "kind": "port",
            "sample": f"oracle fwd+bwd on {info['tiles']} 16x16 tile crops of the same view "
                      f"({info['crop_seconds']} s) plus full-scene projection and binning "
                      f"({info['setup_seconds']} s), extrapolated to the full frame by tile-list work"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    vals = []
    info = None
    for _ in range(max(1, args.warmup)):
        cpu_crop_sample(args, threads, budget_s=2.0)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, info = cpu_crop_sample(args, threads, budget_s=8.0)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = sorted(vals)[len(vals) // 2]
    params_w = args.workload
    ms = 1920 * 1080 / (value * 1e6) * 1e3 if value else None
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "Mpix/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1) if ms else None,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded surface-sampled scene)",
        "config": {"workload": f"{params_w}: mode {args.mode}, distortions {args.distortions}, fwd+bwd",
                   "wall_seconds": round(wall, 1)},
        "cpu_baseline": {"value": round(value, 6), "unit": "Mpix/s", "cores": threads, "kind": "port",
                         "sample": f"oracle (Torch-provider restatement) on tile crops, {info}"},
        "e2e": {"value": round(value, 6), "unit": "Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.impl == "reference":
        res = run_reference(args)
    else:
        res = run_b200(args)
    if res is not None:
        print(json.dumps(res))


if __name__ == "__main__":
    main()
