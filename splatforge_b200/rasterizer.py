"""Host orchestration of the B200 rasterizer: autograd functions over the C ABI.

The differentiable path mirrors the Torch provider's composition
(src/splatforge/studio/batched_renderer.py:45-410):

    (means, quats, scales, opacities, sh)
        --_Project-->  projected means [N,2] (a real autograd intermediate, so
                       ``retain_grad()`` works), radii [N], Gaussian records [N,20]
        --binning-->   per-tile Gaussian lists (device radix sort, one host read of
                       the intersection count)
        --_Raster-->   the nine RenderOutput images

The records tensor carries the per-Gaussian values the tile kernels read (projected
mean, conic, opacity, colour, mode extras); its adjoint is produced by the raster
backward kernel and consumed by the projection backward kernel.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib
from ._lib import L1_SAMPLE_FLOATS, PIXEL_STATE_FLOATS, RECORD_FLOATS, Camera, Settings, call

TILE = 16
# transmittance floor of AmbiSuR renders with distortions: 1e-30 x (far = 1e4)^2 bounds the
# skipped tail's share of L2 by 1e-22, and the floor keeps the final transmittance (kept in
# float32 for the backward, which recovers each sample's transmittance from it by
# division) far above float32 underflow
AMBISUR_DISTORTION_FLOOR = 1e-30

# Optional instrumentation used by bench.py: when PROFILE is a dict, CUDA events are
# recorded on the launching stream around the raster forward / backward calls and
# the (start, end) pairs appended to PROFILE["fwd"] / PROFILE["bwd"].
PROFILE = None
# largest per-pixel L1 sample count seen, per image size (capacity of the next render)
_L1_SEEN = {}
# intersection capacity per (Gaussian count, image size), learned from earlier renders
_ISECT_SEEN = {}
# renders whose L1 samples overflowed the fixed capacity and were rerun with exact
# offsets; renders whose intersections overflowed the learned capacity and were re-binned
COUNTERS = {"l1_reruns": 0, "bin_reruns": 0}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def camera_struct(camera):
    """``Camera`` (src/splatforge/studio/cameras.py:8-22) -> the C ``sf_camera``.

    ``inv(K)`` and the camera centre ``inv(world_to_camera)[:3, 3]`` are evaluated on the
    host in float32, as the reference's CPU path does.
    """
    K = camera.K.detach().to("cpu", torch.float32)
    W = camera.world_to_camera.detach().to("cpu", torch.float32)
    Kinv = torch.linalg.inv(K)
    origin = torch.linalg.inv(W)[:3, 3]
    c = Camera()
    c.R[:] = W[:3, :3].reshape(-1).tolist()
    c.t[:] = W[:3, 3].tolist()
    c.K[:] = K.reshape(-1).tolist()
    c.Kinv[:] = Kinv.reshape(-1).tolist()
    c.origin[:] = origin.tolist()
    c.width = int(camera.width)
    c.height = int(camera.height)
    return c


@dataclass
class RasterSettings:
    """Render-time configuration (RenderConfig fields of src/splatforge/studio/config.py:29-40)."""

    mode: str = "gof"
    distortions: str = "both"
    sigma_extent: float = 3.0
    trunc_sigma: float = 2.0
    eps2d: float = 0.3
    near: float = 0.01
    far: float = 10000.0
    background: tuple = (1.0, 1.0, 1.0)
    antialiased: bool = False
    tile_size: int = 16
    # a pixel stops compositing once its transmittance falls below this floor; the skipped
    # tail changes any weight sum by less than the floor.  AmbiSuR renders that include a
    # distortion stop only at AMBISUR_DISTORTION_FLOOR: their plane depths plane / (n . ray)
    # reach the far plane at grazing angles, so the tail's share of L1 / L2 (linear /
    # quadratic in depth) is bounded by floor x far^2 only
    transmittance_floor: float = 1e-6
    # per-pixel L1 sample capacity of the first forward attempt; None adapts to the
    # largest count seen for this image size (a pixel over capacity triggers an exact
    # per-pixel-offset rerun, so the value only affects speed and memory)
    l1_capacity: int | None = None

    def extent(self):
        return self.trunc_sigma if self.mode == "ambisur" else self.sigma_extent

    def struct(self, sh_degree, sh_coeffs):
        if self.mode not in _lib.MODE:
            raise ValueError(f"unsupported rendering mode: {self.mode}")
        if self.distortions not in _lib.DISTORTIONS:
            raise ValueError("distortions must explicitly be none, l1, l2 or both")
        if self.tile_size != TILE:
            raise ValueError("the B200 rasterizer uses 16x16 tiles")
        s = Settings()
        s.mode = _lib.MODE[self.mode]
        s.distortions = _lib.DISTORTIONS[self.distortions]
        s.tile_size = TILE
        s.sh_degree = int(sh_degree)
        s.sh_coeffs = int(sh_coeffs)
        s.antialiased = int(bool(self.antialiased))
        ext = float(self.extent())
        s.extent = ext
        s.extent_sq = float(torch.tensor(ext**2, dtype=torch.float32))
        s.eps2d = float(self.eps2d)
        s.near_plane = float(self.near)
        s.far_plane = float(self.far)
        s.background[:] = [float(v) for v in self.background]
        s.t_stop = (AMBISUR_DISTORTION_FLOOR if (self.mode == "ambisur" and self.distortions != "none")
                    else float(self.transmittance_floor))
        return s


@dataclass
class _Plan:
    cam: Camera
    settings: Settings
    n: int
    device: torch.device
    selected: torch.Tensor | None = None
    rect: torch.Tensor | None = None
    count: torch.Tensor | None = None
    depth_key: torch.Tensor | None = None
    nonfinite: torch.Tensor | None = None
    ids: torch.Tensor | None = None
    ranges: torch.Tensor | None = None
    n_isect: int = 0
    # bounded binning: (order, offsets, overflow flag) until the forward's read-back
    pending: tuple | None = None
    absgrad: torch.Tensor | None = None
    l1_capacity: int | None = None
    error_word: torch.Tensor | None = None
    stats: dict = field(default_factory=dict)

    @property
    def tiles_x(self):
        return (self.cam.width + TILE - 1) // TILE

    @property
    def n_tiles(self):
        return self.tiles_x * ((self.cam.height + TILE - 1) // TILE)


def _check_inputs(tensors, names):
    dev = tensors[0].device
    if dev.type != "cuda":
        raise ValueError("the B200 rasterizer requires CUDA tensors; there is no CPU fallback")
    for t, name in zip(tensors, names):
        if t.dtype != torch.float32:
            raise ValueError(f"{name}: the B200 rasterizer requires float32 (got {t.dtype})")
        if t.device != dev:
            raise ValueError("tensor dtype/device must match explicitly")
    return dev


class _Project(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, opacities, sh, plan):
        n = plan.n
        dev = plan.device
        means, quats, scales, opacities, sh = (
            t.contiguous() for t in (means, quats, scales, opacities, sh)
        )
        means2d = torch.empty((n, 2), device=dev, dtype=torch.float32)
        radii = torch.empty((n,), device=dev, dtype=torch.float32)
        records = torch.empty((n, RECORD_FLOATS), device=dev, dtype=torch.float32)
        plan.rect = torch.empty((n, 4), device=dev, dtype=torch.int32)
        plan.count = torch.empty((n,), device=dev, dtype=torch.int32)
        plan.depth_key = torch.empty((n,), device=dev, dtype=torch.int32)
        plan.nonfinite = torch.zeros((1,), device=dev, dtype=torch.int32)
        call(
            "sf_b200_project_forward",
            _ptr(means), _ptr(quats), _ptr(scales), _ptr(opacities), _ptr(sh), _ptr(plan.selected),
            n, ctypes.byref(plan.cam), ctypes.byref(plan.settings),
            _ptr(means2d), _ptr(radii), _ptr(records), _ptr(plan.rect), _ptr(plan.count),
            _ptr(plan.depth_key), _ptr(plan.nonfinite), _stream(dev),
        )
        ctx.save_for_backward(means, quats, scales, opacities, sh)
        ctx.plan = plan
        ctx.mark_non_differentiable(radii)
        return means2d, radii, records

    @staticmethod
    def backward(ctx, g_means2d, g_radii, g_records):
        means, quats, scales, opacities, sh = ctx.saved_tensors
        plan = ctx.plan
        n, dev = plan.n, plan.device
        g_means2d = (
            torch.zeros((n, 2), device=dev) if g_means2d is None else g_means2d.contiguous()
        )
        g_records = (
            torch.zeros((n, RECORD_FLOATS), device=dev)
            if g_records is None
            else g_records.contiguous()
        )
        need = ctx.needs_input_grad
        outs = [
            torch.empty_like(t) if need[i] else None
            for i, t in enumerate((means, quats, scales, opacities, sh))
        ]
        call(
            "sf_b200_project_backward",
            _ptr(means), _ptr(quats), _ptr(scales), _ptr(opacities), _ptr(sh), n,
            ctypes.byref(plan.cam), ctypes.byref(plan.settings), _ptr(g_means2d), _ptr(g_records),
            *(_ptr(o) for o in outs), _stream(dev),
        )
        return (*outs, None)


def _size_class(n):
    """Round a buffer length up to one of eight classes per octave (<= 12.5% larger).

    The per-render buffers whose size follows the pose (intersection ids, the binning
    workspace) then come from a small set of sizes, so the caching allocator finds an
    exact-size cached block for a pose it has seen before instead of splitting blocks
    until a request needs a fresh device allocation."""
    if n <= 1 << 20:
        return n
    step = 1 << (n.bit_length() - 4)
    return (n + step - 1) // step * step


def _class_empty(n, dtype, dev):
    return torch.empty((_size_class(n),), device=dev, dtype=dtype)[:n]


_PINNED = {}


def _pinned_scratch(dtype=torch.int64):
    """A small pinned host buffer for the synchronous read-backs (per thread, per dtype)."""
    import threading

    key = (threading.get_ident(), dtype)
    buf = _PINNED.get(key)
    if buf is None:
        buf = torch.empty((4,), dtype=dtype, pin_memory=True)
        _PINNED[key] = buf
    return buf


def _isect_capacity(total):
    """Intersection capacity for a count: 1.2x, in the allocator's size classes."""
    return _size_class(int(total * 1.2) + 1024)


def bin_gaussians(plan):
    """Device tile binning.

    The first render of a (Gaussian count, image size) reads the intersection count
    back (one host synchronisation) and sizes the lists exactly.  Later renders size
    them by the capacity learned from the earlier ones and read nothing back here: the
    count sits on the device (offsets[n]) for ``sf_b200_bin_emit_bounded``, and the
    count, the non-finite flag and the overflow flag come back with the raster
    forward's one read-back (``_Raster.forward``), which re-bins exactly and reruns the
    forward if the capacity was exceeded."""
    n, dev = plan.n, plan.device
    size = ctypes.c_size_t()
    call("sf_b200_bin_workspace_bytes", n, 0, plan.n_tiles, ctypes.byref(size))
    ws = _class_empty(max(size.value, 1), torch.uint8, dev)
    order = torch.empty((n,), device=dev, dtype=torch.int32)
    offsets = torch.empty((n + 1,), device=dev, dtype=torch.int64)
    call(
        "sf_b200_bin_order", _ptr(plan.count), _ptr(plan.depth_key), n, _ptr(order), _ptr(offsets),
        _ptr(ws), size.value, _stream(dev),
    )
    plan.ranges = torch.empty((plan.n_tiles, 2), device=dev, dtype=torch.int32)
    cap = _ISECT_SEEN.get((n, plan.cam.width, plan.cam.height))
    if cap is None:
        # the read-back: two small async copies into pinned memory
        host, host32 = _pinned_scratch(), _pinned_scratch(torch.int32)
        host[0:1].copy_(offsets[n:n + 1], non_blocking=True)
        host32[0:1].copy_(plan.nonfinite[0:1], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        if int(host32[0]):
            raise FloatingPointError("non-finite projected bounds")
        _emit_exact(plan, order, offsets, int(host[0]))
        return plan
    call("sf_b200_bin_workspace_bytes", n, cap, plan.n_tiles, ctypes.byref(size))
    if size.value > ws.numel():
        ws = _class_empty(size.value, torch.uint8, dev)
    plan.ids = _class_empty(cap, torch.int32, dev)
    overflow = torch.zeros((1,), device=dev, dtype=torch.int32)
    call(
        "sf_b200_bin_emit_bounded", _ptr(order), _ptr(offsets), _ptr(plan.rect), n, cap,
        plan.tiles_x, plan.n_tiles, _ptr(plan.ids), _ptr(plan.ranges), _ptr(ws), size.value,
        _ptr(overflow), _stream(dev),
    )
    plan.pending = (order, offsets, overflow)
    return plan


def _emit_exact(plan, order, offsets, total):
    n, dev = plan.n, plan.device
    plan.n_isect = int(total)
    _ISECT_SEEN[(n, plan.cam.width, plan.cam.height)] = _isect_capacity(total)
    size = ctypes.c_size_t()
    call("sf_b200_bin_workspace_bytes", n, plan.n_isect, plan.n_tiles, ctypes.byref(size))
    ws = _class_empty(max(size.value, 1), torch.uint8, dev)
    plan.ids = _class_empty(max(plan.n_isect, 1), torch.int32, dev)
    call(
        "sf_b200_bin_emit", _ptr(order), _ptr(offsets), _ptr(plan.rect), n, plan.n_isect,
        plan.tiles_x, plan.n_tiles, _ptr(plan.ids), _ptr(plan.ranges), _ptr(ws), size.value,
        _stream(dev),
    )


def _settle_binning(plan, needed):
    """The forward's one read-back: the largest L1 sample count (when ``needed``) and,
    after bounded binning, the intersection count and the non-finite and overflow
    flags.  Returns (largest L1 count or 0, whether the lists were re-binned)."""
    dev = plan.device
    host, host32 = _pinned_scratch(), _pinned_scratch(torch.int32)
    if needed is not None:
        host32[1:2].copy_(needed, non_blocking=True)
    if plan.pending is not None:
        order, offsets, overflow = plan.pending
        host[0:1].copy_(offsets[plan.n:plan.n + 1], non_blocking=True)
        host32[0:1].copy_(plan.nonfinite[0:1], non_blocking=True)
        host32[2:3].copy_(overflow, non_blocking=True)
    torch.cuda.current_stream(dev).synchronize()
    most = int(host32[1]) if needed is not None else 0
    if plan.pending is None:
        return most, False
    order, offsets, _ = plan.pending
    plan.pending = None
    if int(host32[0]):
        raise FloatingPointError("non-finite projected bounds")
    total = int(host[0])
    key = (plan.n, plan.cam.width, plan.cam.height)
    if int(host32[2]):
        # the learned capacity was too small: exact lists, and the caller reruns
        COUNTERS["bin_reruns"] += 1
        _emit_exact(plan, order, offsets, total)
        return most, True
    plan.n_isect = total
    if _isect_capacity(total) > _ISECT_SEEN.get(key, 0):
        _ISECT_SEEN[key] = _isect_capacity(total)
    return most, False


class _Raster(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2d, records, plan):
        dev = plan.device
        H, W = plan.cam.height, plan.cam.width
        f = dict(device=dev, dtype=torch.float32)
        rgb = torch.empty((H, W, 3), **f)
        alpha = torch.empty((H, W, 1), **f)
        depth = torch.empty((H, W, 1), **f)
        normals = torch.empty((H, W, 3), **f)
        l1 = torch.empty((H, W, 1), **f)
        l2 = torch.empty((H, W, 1), **f)
        median = torch.empty((H, W, 1), **f)
        ray_color = torch.empty((H, W, 1), **f)
        amb = torch.empty((H, W, 1), **f)
        state = torch.empty((H * W, PIXEL_STATE_FLOATS), **f)
        records = records.contiguous()
        use_l1 = bool(plan.settings.distortions & 1)
        l1s, l1_off, cap, slots = None, None, 0, 0
        needed = None
        key = (W, H)
        if use_l1:
            if plan.l1_capacity is not None:
                cap = int(plan.l1_capacity)
            else:
                cap = _L1_SEEN.get(key, 256)
            cap = max(32, (cap + 31) // 32 * 32)
            slots = plan.n_tiles * TILE * TILE * cap
            l1s = torch.empty((L1_SAMPLE_FLOATS, slots), **f)
            needed = torch.zeros((1,), device=dev, dtype=torch.int32)
        counters = torch.zeros((2,), device=dev, dtype=torch.int64) if PROFILE is not None else None

        def run():
            call(
                "sf_b200_raster_forward", _ptr(records), plan.n, _ptr(plan.ids), _ptr(plan.ranges),
                ctypes.byref(plan.cam), ctypes.byref(plan.settings),
                _ptr(rgb), _ptr(alpha), _ptr(depth), _ptr(normals), _ptr(l1), _ptr(l2), _ptr(median),
                _ptr(ray_color), _ptr(amb), _ptr(state), _ptr(l1s), slots, _ptr(l1_off), cap,
                _ptr(needed), _ptr(counters), _stream(dev),
            )

        if PROFILE is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
            run()
            ev[1].record()
            PROFILE["fwd"].append(ev)
            PROFILE.setdefault("counters", []).append(counters)
        else:
            run()
        if use_l1 or plan.pending is not None:
            most, rebinned = _settle_binning(plan, needed)
            if rebinned:
                plan.stats["bin_rerun"] = True
                if needed is not None:
                    needed.zero_()
                run()
                if use_l1:
                    most, _ = _settle_binning(plan, needed)
        if use_l1:
            plan.stats["l1_max_samples"] = most
            plan.stats["l1_capacity"] = cap
            if plan.l1_capacity is None:
                # capacity of the next render of this size: at least 1.2x the largest count
                # seen; it never shrinks and grows by at least half each time it must, so a
                # sequence of poses settles on one capacity (one buffer size) quickly
                want = int(most * 1.2 + 31) // 32 * 32
                current = _L1_SEEN.get(key, 0)
                if want > current:
                    _L1_SEEN[key] = max(want, (current * 3 // 2 + 63) // 64 * 64)
            if most > cap:
                # capacity exceeded somewhere: exact per-pixel (CSR) storage and a rerun
                plan.stats["l1_rerun"] = True
                COUNTERS["l1_reruns"] += 1
                ws_bytes = (H * W + 2048) * 8 + H * W * 4 + 4096
                ws = torch.empty((ws_bytes,), device=dev, dtype=torch.uint8)
                l1_off = torch.empty((H * W + 1,), device=dev, dtype=torch.int64)
                call("sf_b200_l1_offsets", ctypes.byref(plan.cam), _ptr(state), _ptr(l1_off),
                     _ptr(ws), ws_bytes, _stream(dev))
                slots = int(l1_off[H * W].item())
                l1s = torch.empty((L1_SAMPLE_FLOATS, max(slots, 1)), **f)
                run()
            call(
                "sf_b200_l1_resolve", ctypes.byref(plan.cam), ctypes.byref(plan.settings), _ptr(state),
                _ptr(l1s), slots, _ptr(l1_off), cap, most, _ptr(l1), _stream(dev),
            )
        # the pixel state and the L1 sample store are saved tensors, so autograd frees
        # them once the backward has run (a caller that keeps the outputs of one view
        # while rendering the next then holds one L1 store, not two)
        ctx.save_for_backward(records, state, l1s, l1_off)
        ctx.plan = plan
        ctx.l1 = (slots, cap)
        return rgb, alpha, depth, normals, l1, l2, median, ray_color, amb

    @staticmethod
    def backward(ctx, g_rgb, g_alpha, g_depth, g_normals, g_l1, g_l2, g_median, g_var, g_amb):
        records, state, l1s, l1_off = ctx.saved_tensors
        plan = ctx.plan
        dev, n = plan.device, plan.n
        grads = [
            None if g is None else g.contiguous()
            for g in (g_rgb, g_alpha, g_depth, g_normals, g_l1, g_l2, g_median, g_var, g_amb)
        ]
        grad_records = torch.zeros((n, RECORD_FLOATS), device=dev, dtype=torch.float32)
        grad_means2d = torch.empty((n, 2), device=dev, dtype=torch.float32)
        absgrad = plan.absgrad if plan.absgrad is not None else torch.zeros((n, 2), device=dev)
        slots, cap = ctx.l1
        ev = None
        if PROFILE is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        plan.error_word = torch.zeros((1,), device=dev, dtype=torch.int32)
        call(
            "sf_b200_raster_backward", _ptr(records), n, _ptr(plan.ids), _ptr(plan.ranges),
            ctypes.byref(plan.cam), ctypes.byref(plan.settings), _ptr(state), _ptr(l1s), slots,
            _ptr(l1_off), cap, *(_ptr(g) for g in grads), _ptr(grad_records), _ptr(grad_means2d),
            _ptr(absgrad), _ptr(plan.error_word), _stream(dev),
        )
        if ev is not None:
            ev[1].record()
            PROFILE["bwd"].append(ev)
        return grad_means2d, grad_records, None


def kernel_launches():
    """Kernels launched so far by libsf_b200.so in this process."""
    return int(_lib.lib().sf_b200_kernel_launches())


def rasterize(means, quats, scales, opacities, sh, sh_degree, camera, settings, *, selected=None):
    """One differentiable render.  Returns a dict of the nine images plus
    ``projected_means`` (with ``.absgrad`` when it requires grad) and ``projected_radii``."""
    dev = _check_inputs((means, quats, scales, opacities, sh), ("means", "quats", "scales", "opacities", "sh"))
    n = means.shape[0]
    if sh.ndim != 3 or sh.shape[0] != n or sh.shape[2] != 3:
        raise ValueError("sh must be [N, K, 3]")
    with torch.cuda.device(dev):
        plan = _Plan(camera_struct(camera), settings.struct(sh_degree, sh.shape[1]), n, dev)
        plan.l1_capacity = settings.l1_capacity
        if selected is not None:
            plan.selected = selected.to(device=dev, dtype=torch.uint8).contiguous()
        means2d, radii, records = _Project.apply(means, quats, scales, opacities, sh, plan)
        if means2d.requires_grad:
            means2d.retain_grad()
            means2d.absgrad = torch.zeros_like(means2d)
            plan.absgrad = means2d.absgrad
        bin_gaussians(plan)
        images = _Raster.apply(means2d, records, plan)
    names = ("rgb", "alpha", "depth", "normals", "distortion_l1", "distortion_l2",
             "median_depth", "ray_color", "ambiguity_mask")
    out = dict(zip(names, images))
    out["projected_means"] = means2d
    out["projected_radii"] = radii
    out["n_isect"] = plan.n_isect
    out["stats"] = plan.stats
    out["plan"] = plan
    return out
