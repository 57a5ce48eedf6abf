"""Operator runners with the Torch provider's signatures, backed by libsf_b200.so.

Each runner takes exactly the positional tensors and keyword attributes SplatForge's
operator validator passes (src/splatforge/gaussian/ops.py:23-51, 54-172) and returns
what the Torch provider's function returns:

* ``covariance(quats, scales)``                      gaussian.covariance@1 (reference.py:33-35)
* ``sh_color(coefficients, directions, *, degree)``  gaussian.sh_color@1   (reference.py:85-113)
* ``alpha_composite_selected(alphas, colors, depths, normals, *, distortions)``
                                                     splat.alpha_composite@3 (reference.py:182-186)
* ``opacity_field(points, means, inverse_covariances, opacities, origins, *, gaussian_chunk)``
                                                     gaussian.opacity_field@1 (reference.py:194-222)
* ``patch_zncc(a, b, mask, *, epsilon)``             matching.patch_zncc@1 (reference.py:225-236)
* ``sh_ambiguity(coefficients)``                     gaussian.sh_ambiguity@1 (reference.py:116-117)
* ``ray_color_variance(w, c, composite)`` / ``ray_color_variance_batch(...)``
                                                     gaussian.ray_color_variance@1/@2 (reference.py:120-122, 189-191)

They accept CUDA float32 tensors only and raise ``ValueError`` otherwise, like the
reference's CUDA composite provider (cuda_composite.py:79-85); nothing falls back
to Torch.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import call
from .rasterizer import _ptr, _stream


def _require_cuda_f32(name, *tensors):
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda" or t.dtype != torch.float32:
            raise ValueError(f"{name} requires explicit CUDA float32 tensors (no fallback)")
    dev = tensors[0].device
    if any(t.device != dev for t in tensors):
        raise ValueError(f"{name}: tensors must share one device")
    return dev


# ---------------------------------------------------------------- gaussian.covariance@1
class _Covariance(torch.autograd.Function):
    @staticmethod
    def forward(ctx, quats, scales):
        dev = quats.device
        q, s = quats.contiguous(), scales.contiguous()
        n = q.shape[0]
        cov = torch.empty((n, 3, 3), device=dev, dtype=torch.float32)
        call("sf_b200_covariance_forward", _ptr(q), _ptr(s), n, _ptr(cov), _stream(dev))
        ctx.save_for_backward(q, s)
        return cov

    @staticmethod
    def backward(ctx, g):
        q, s = ctx.saved_tensors
        dev = q.device
        gq = torch.empty_like(q) if ctx.needs_input_grad[0] else None
        gs = torch.empty_like(s) if ctx.needs_input_grad[1] else None
        call("sf_b200_covariance_backward", _ptr(q), _ptr(s), q.shape[0], _ptr(g.contiguous()), _ptr(gq), _ptr(gs),
             _stream(dev))
        return gq, gs


def covariance(quats, scales):
    with torch.cuda.device(_require_cuda_f32("gaussian.covariance@1", quats, scales)):
        return _Covariance.apply(quats, scales)


# ---------------------------------------------------------------- gaussian.sh_color@1
class _ShColor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, coeffs, dirs, degree):
        dev = coeffs.device
        c, d = coeffs.contiguous(), dirs.contiguous()
        n, K = c.shape[0], c.shape[1]
        out = torch.empty((n, 3), device=dev, dtype=torch.float32)
        call("sf_b200_sh_color_forward", _ptr(c), K, _ptr(d), n, degree, _ptr(out), _stream(dev))
        ctx.save_for_backward(c, d)
        ctx.degree = degree
        return out

    @staticmethod
    def backward(ctx, g):
        c, d = ctx.saved_tensors
        dev = c.device
        gc = torch.empty_like(c) if ctx.needs_input_grad[0] else None
        gd = torch.empty_like(d) if ctx.needs_input_grad[1] else None
        call("sf_b200_sh_color_backward", _ptr(c), c.shape[1], _ptr(d), c.shape[0], ctx.degree, _ptr(g.contiguous()),
             _ptr(gc), _ptr(gd), _stream(dev))
        return gc, gd, None


def sh_color(coefficients, directions, *, degree):
    with torch.cuda.device(_require_cuda_f32("gaussian.sh_color@1", coefficients, directions)):
        return _ShColor.apply(coefficients, directions, int(degree))


# ---------------------------------------------------------------- splat.alpha_composite@3
class _Composite(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, c, d, n, dist):
        dev = a.device
        a, c, d, n = (t.contiguous() for t in (a, c, d, n))
        B, N, P = a.shape
        f = dict(device=dev, dtype=torch.float32)
        rgb = torch.empty((B, P, 3), **f)
        alpha = torch.empty((B, P), **f)
        znum = torch.empty((B, P), **f)
        nnum = torch.empty((B, P, 3), **f)
        l1 = torch.empty((B, P), **f)
        l2 = torch.empty((B, P), **f)
        median = torch.empty((B, P), **f)
        w = torch.empty((B, N, P), **f)
        size = ctypes.c_size_t()
        call("sf_b200_composite_workspace_bytes", B, N, P, dist, ctypes.byref(size))
        ws = torch.empty((size.value,), device=dev, dtype=torch.uint8)
        call("sf_b200_alpha_composite_forward", _ptr(a), _ptr(c), _ptr(d), _ptr(n), B, N, P, dist, _ptr(rgb),
             _ptr(alpha), _ptr(znum), _ptr(nnum), _ptr(l1), _ptr(l2), _ptr(median), _ptr(w), _ptr(ws), size.value,
             _stream(dev))
        ctx.save_for_backward(a, c, d, n, w, ws)
        ctx.dist = dist
        ctx.set_materialize_grads(False)
        return rgb, alpha, znum, nnum, l1, l2, median, w

    @staticmethod
    def backward(ctx, g_rgb, g_alpha, g_znum, g_nnum, g_l1, g_l2, g_median, g_w):
        a, c, d, n, w, ws = ctx.saved_tensors
        dev = a.device
        B, N, P = a.shape
        grads = [None if g is None else g.contiguous() for g in (g_rgb, g_alpha, g_znum, g_nnum, g_l1, g_l2, g_median, g_w)]
        da, dc, dd, dn = (torch.empty_like(t) for t in (a, c, d, n))
        call("sf_b200_alpha_composite_backward", _ptr(a), _ptr(c), _ptr(d), _ptr(n), B, N, P, ctx.dist, _ptr(w),
             _ptr(ws), ws.numel(), *(_ptr(g) for g in grads), _ptr(da), _ptr(dc), _ptr(dd), _ptr(dn), _stream(dev))
        return da, dc, dd, dn, None


def alpha_composite_selected(alphas, colors, depths, normals, *, distortions):
    if distortions not in _lib.DISTORTIONS:
        raise ValueError("distortions must explicitly be none, l1, l2 or both")
    dev = _require_cuda_f32("splat.alpha_composite@3", alphas, colors, depths, normals)
    with torch.cuda.device(dev):
        return _Composite.apply(alphas, colors, depths, normals, _lib.DISTORTIONS[distortions])


def alpha_composite_batch(alphas, colors, depths, normals):
    """``splat.alpha_composite@2``: the batched composite with both distortion terms
    (reference.py:151-179), the @3 kernel with distortions "both"."""
    dev = _require_cuda_f32("splat.alpha_composite@2", alphas, colors, depths, normals)
    with torch.cuda.device(dev):
        return _Composite.apply(alphas, colors, depths, normals, _lib.DISTORTIONS["both"])


def alpha_composite(alphas, colors, depths, normals):
    """``splat.alpha_composite@1``: one front-to-back composite, alphas [N,P], colors
    [N,3], depths [N,P], normals [N,P,3] (reference.py:125-148); the same 8-tuple without
    the batch axis."""
    outs = alpha_composite_batch(alphas[None], colors[None], depths[None], normals[None])
    return tuple(o[0] for o in outs)


# ---------------------------------------------------------------- gaussian.opacity_field@1
# Two implementations: ``opacity_field`` evaluates every (point, Gaussian, origin)
# triple and never synchronises; ``opacity_field_culled`` walks per-view candidate
# lists (for the exporter's large grids) and synchronises once per origin, which its
# manifest declares.
# contributions at or below this are dropped by the culled kernel
FIELD_CUTOFF = 1e-7
FIELD_FACE_CELLS = 128
# per-view candidate pairs above this make the runner coarsen the cube map instead
FIELD_PAIR_LIMIT = 1 << 28
_FIELD_WS = {}   # device index -> workspace tensor
_FIELD_CFG = {}  # (device, N, P, requested face_cells) -> (face_cells, max_pairs) that fit


def opacity_field(points, means, inverse_covariances, opacities, origins, *, gaussian_chunk=1024):
    """Forward only (the manifest declares ``backward: false``).  ``gaussian_chunk``
    only affects the reference's memory use; the field does not depend on it."""
    dev = _require_cuda_f32("gaussian.opacity_field@1", points, means, inverse_covariances, opacities, origins)
    del gaussian_chunk
    if origins.shape[0] < 1:
        raise ValueError("opacity field requires at least one origin")
    with torch.cuda.device(dev), torch.no_grad():
        p, m, q, o, org = (t.contiguous() for t in (points, means, inverse_covariances, opacities, origins))
        out = torch.empty((p.shape[0],), device=dev, dtype=torch.float32)
        size = ctypes.c_size_t()
        call("sf_b200_opacity_field_workspace_bytes", m.shape[0], ctypes.byref(size))
        ws = torch.empty((size.value,), device=dev, dtype=torch.uint8)
        call("sf_b200_opacity_field", _ptr(p), p.shape[0], _ptr(m), _ptr(q), _ptr(o), m.shape[0], _ptr(org),
             org.shape[0], _ptr(out), _ptr(ws), size.value, _stream(dev))
    return out


def opacity_field_culled(points, means, inverse_covariances, opacities, origins, *, gaussian_chunk=1024,
                         cutoff=FIELD_CUTOFF, face_cells=None, stats=None):
    """The opacity field through per-view cube-map candidate lists: contributions at or
    below ``cutoff`` are dropped, everything else is evaluated as in the brute-force
    kernel.  The cube-map resolution (``face_cells``, default FIELD_FACE_CELLS, lowered
    when a view's candidate lists would exceed FIELD_PAIR_LIMIT) and the list capacity
    are remembered per problem shape, and the workspace is kept per device.  With a
    ``stats`` dict, ``stats["pairs_evaluated"]`` and ``stats["query_ms"]`` accumulate the
    evaluated (query, candidate) pairs and the query kernels' CUDA-event time."""
    dev = _require_cuda_f32("gaussian.opacity_field@1", points, means, inverse_covariances, opacities, origins)
    del gaussian_chunk
    if origins.shape[0] < 1:
        raise ValueError("opacity field requires at least one origin")
    with torch.cuda.device(dev), torch.no_grad():
        p, m, q, o, org = (t.contiguous() for t in (points, means, inverse_covariances, opacities, origins))
        n, npts = m.shape[0], p.shape[0]
        out = torch.empty((npts,), device=dev, dtype=torch.float32)
        shape = (dev.index, n, npts, face_cells)
        cells, pairs = _FIELD_CFG.get(shape, (face_cells or FIELD_FACE_CELLS, 64 * max(n, 1)))
        needed = ctypes.c_int64()
        for _ in range(8):
            size = ctypes.c_size_t()
            call("sf_b200_opacity_field_culled_workspace_bytes", npts, n, pairs, cells, ctypes.byref(size))
            ws = _FIELD_WS.get(dev.index)
            if ws is None or ws.numel() < size.value:
                _FIELD_WS.pop(dev.index, None)
                ws = torch.empty((size.value,), device=dev, dtype=torch.uint8)
                _FIELD_WS[dev.index] = ws
            args = (_ptr(p), npts, _ptr(m), _ptr(q), _ptr(o), n, _ptr(org), org.shape[0], ctypes.c_float(cutoff),
                    cells, _ptr(out), _ptr(ws), ws.numel(), pairs, ctypes.byref(needed))
            if stats is None:
                status = _lib.lib().sf_b200_opacity_field_culled(*args, _stream(dev))
            else:
                counter = torch.zeros((1,), device=dev, dtype=torch.int64)
                qms = ctypes.c_float(0.0)
                status = _lib.lib().sf_b200_opacity_field_culled_stats(*args, _ptr(counter), ctypes.byref(qms),
                                                                        _stream(dev))
            if status == _lib.SF_OK:
                _FIELD_CFG[shape] = (cells, pairs)
                if stats is not None:
                    stats["pairs_evaluated"] = stats.get("pairs_evaluated", 0) + int(counter.item())
                    stats["query_ms"] = stats.get("query_ms", 0.0) + float(qms.value)
                return out
            if status != _lib.SF_ERR_CAPACITY or needed.value <= pairs:
                raise _lib.NativeError(_lib.lib().sf_b200_last_error().decode())
            if needed.value > FIELD_PAIR_LIMIT and cells > 8 and face_cells is None:
                # fewer, larger cells: pairs scale with the square of the face resolution
                cells = max(8, int(cells * 0.97 * (FIELD_PAIR_LIMIT / needed.value) ** 0.5))
                pairs = FIELD_PAIR_LIMIT
            else:
                pairs = int(needed.value * 1.1) + 1024
        raise _lib.NativeError("opacity_field_culled: candidate lists did not fit after resizing")


class OpacityFieldPlan:
    """Repeated evaluations of ``gaussian.opacity_field@1`` against one Gaussian set and
    one set of origins, as the GOF exporter makes them (the grid, then every bisection
    step, src/splatforge/studio/exporters.py:56-88): every view's culled candidate lists
    are built once (one host synchronisation per origin); each call then evaluates its
    queries for all views at once, with no host synchronisation.  The values equal
    ``opacity_field_culled``'s for the same ``cutoff`` and ``face_cells``."""

    def __init__(self, means, inverse_covariances, opacities, origins, *, cutoff=FIELD_CUTOFF, face_cells=None):
        dev = _require_cuda_f32("gaussian.opacity_field@1", means, inverse_covariances, opacities, origins)
        if origins.shape[0] < 1:
            raise ValueError("opacity field requires at least one origin")
        self.device = dev
        self.n = means.shape[0]
        self.origins = origins.contiguous()
        nc = self.origins.shape[0]
        F = face_cells or FIELD_FACE_CELLS
        total = most = 0
        needed = (ctypes.c_int64 * 2)()
        with torch.cuda.device(dev), torch.no_grad():
            m, q, o = (t.contiguous() for t in (means, inverse_covariances, opacities))
            for _ in range(8):
                size = ctypes.c_size_t()
                call("sf_b200_opacity_field_plan_bytes", self.n, nc, F, total, most, ctypes.byref(size))
                plan = torch.empty((max(size.value, 1),), device=dev, dtype=torch.uint8)
                status = _lib.lib().sf_b200_opacity_field_plan_build(
                    _ptr(m), _ptr(q), _ptr(o), self.n, _ptr(self.origins), nc, ctypes.c_float(cutoff), F, _ptr(plan),
                    plan.numel(), total, most, needed, _stream(dev))
                if status == _lib.SF_OK:
                    break
                if status != _lib.SF_ERR_CAPACITY:
                    raise _lib.NativeError(_lib.lib().sf_b200_last_error().decode())
                if needed[1] > FIELD_PAIR_LIMIT and F > 8 and face_cells is None:
                    # fewer, larger cells: pairs scale with the square of the face resolution
                    F = max(8, int(F * 0.97 * (FIELD_PAIR_LIMIT / needed[1]) ** 0.5))
                    total = most = 0
                else:
                    total, most = int(needed[0]), int(needed[1])
            else:
                raise _lib.NativeError("opacity field plan: candidate lists did not fit after resizing")
        self.plan, self.face_cells, self.total_pairs, self.max_view_pairs = plan, F, total, most
        self._ws = None

    def __call__(self, points):
        dev = _require_cuda_f32("gaussian.opacity_field@1", points, self.origins)
        if dev != self.device:
            raise ValueError("opacity field plan: points must be on the plan's device")
        nc = self.origins.shape[0]
        with torch.cuda.device(dev), torch.no_grad():
            p = points.contiguous()
            out = torch.empty((p.shape[0],), device=dev, dtype=torch.float32)
            step = (2**31 - 1) // nc
            for start in range(0, p.shape[0], step):
                part = p[start:start + step]
                size = ctypes.c_size_t()
                call("sf_b200_opacity_field_plan_query_bytes", part.shape[0], nc, self.face_cells, ctypes.byref(size))
                if self._ws is None or self._ws.numel() < size.value:
                    self._ws = None
                    self._ws = torch.empty((max(size.value, 1),), device=dev, dtype=torch.uint8)
                call("sf_b200_opacity_field_plan_eval", _ptr(self.plan), self.n, nc, self.face_cells, self.total_pairs,
                     self.max_view_pairs, _ptr(self.origins), _ptr(part), part.shape[0], _ptr(out[start:]),
                     _ptr(self._ws), self._ws.numel(), _stream(dev))
        return out


# ---------------------------------------------------------------- gaussian.sh_ambiguity@1
class _ShAmbiguity(torch.autograd.Function):
    @staticmethod
    def forward(ctx, coeffs):
        dev = coeffs.device
        c = coeffs.contiguous()
        n, K = c.shape[0], c.shape[1]
        out = torch.empty((n,), device=dev, dtype=torch.float32)
        with torch.cuda.device(dev):
            call("sf_b200_sh_ambiguity", _ptr(c), n, K, _ptr(out), _stream(dev))
        ctx.save_for_backward(c)
        return out

    @staticmethod
    def backward(ctx, g):
        (c,) = ctx.saved_tensors
        dev = c.device
        gc = torch.empty_like(c)
        gg = g.contiguous().float()
        with torch.cuda.device(dev):
            call("sf_b200_sh_ambiguity_backward", _ptr(c), c.shape[0], c.shape[1], _ptr(gg), _ptr(gc), _stream(dev))
        return gc


def sh_ambiguity(coefficients):
    """``gaussian.sh_ambiguity@1``: squared norm of the SH coefficients [N,K,3] outside
    the DC band -> [N] (reference.py:116-117); differentiable."""
    _require_cuda_f32("gaussian.sh_ambiguity@1", coefficients)
    return _ShAmbiguity.apply(coefficients)


# ---------------------------------------------------------------- gaussian.ray_color_variance@1/@2
class _RayColorVariance(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weights, colors, composite):
        dev = colors.device
        w, c, r = (t.detach().contiguous() for t in (weights, colors, composite))
        B, N, P = w.shape
        out = torch.empty((B, P), device=dev, dtype=torch.float32)
        with torch.cuda.device(dev):
            call("sf_b200_ray_color_variance", _ptr(w), _ptr(c), _ptr(r), B, N, P, _ptr(out), _stream(dev))
        ctx.save_for_backward(w, c, r)
        return out

    @staticmethod
    def backward(ctx, g):
        w, c, r = ctx.saved_tensors
        dev = c.device
        B, N, P = w.shape
        gc = torch.empty_like(c)
        gg = g.contiguous().float()
        with torch.cuda.device(dev):
            call("sf_b200_ray_color_variance_backward", _ptr(w), _ptr(c), _ptr(r), _ptr(gg), B, N, P, _ptr(gc),
                 _stream(dev))
        return None, gc, None


def ray_color_variance_batch(weights, colors, composite):
    """``gaussian.ray_color_variance@2``: weights [B,N,P], colors [B,N,3], composite [B,P,3]
    -> [B,P] = sum_n stopgrad(w) |c - stopgrad(composite)|^2; only the colours receive
    gradients (reference.py:189-191)."""
    _require_cuda_f32("gaussian.ray_color_variance@2", weights, colors, composite)
    return _RayColorVariance.apply(weights, colors, composite)


def ray_color_variance(weights, colors, composite):
    """``gaussian.ray_color_variance@1``: the single-batch form, weights [N,P], colors
    [N,3], composite [P,3] -> [P] (reference.py:120-122)."""
    _require_cuda_f32("gaussian.ray_color_variance@1", weights, colors, composite)
    return _RayColorVariance.apply(weights[None], colors[None], composite[None])[0]


# ---------------------------------------------------------------- matching.patch_zncc@1
class _PatchZncc(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, mask, epsilon):
        dev = a.device
        S = a.shape[-1]
        rows = a.numel() // S if S else 0
        a2, b2, m2 = (t.contiguous().reshape(rows, S) for t in (a, b, mask))
        corr = torch.empty((rows,), device=dev, dtype=torch.float32)
        valid = torch.empty((rows,), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            call("sf_b200_patch_zncc", _ptr(a2), _ptr(b2), _ptr(m2), rows, S, ctypes.c_float(epsilon), _ptr(corr),
                 _ptr(valid), _stream(dev))
        ctx.save_for_backward(a2, b2, m2)
        ctx.shape, ctx.epsilon = a.shape, epsilon
        ctx.mark_non_differentiable(valid)
        return corr.reshape(a.shape[:-1]), valid.bool().reshape(a.shape[:-1])

    @staticmethod
    def backward(ctx, g_corr, g_valid):
        a2, b2, m2 = ctx.saved_tensors
        rows, S = a2.shape
        if g_corr is None:
            return None, None, None, None
        dev = a2.device
        g = g_corr.contiguous().reshape(rows).float()
        ga = torch.empty_like(a2)
        gb = torch.empty_like(b2)
        with torch.cuda.device(dev):
            call("sf_b200_patch_zncc_backward", _ptr(a2), _ptr(b2), _ptr(m2), rows, S, ctypes.c_float(ctx.epsilon),
                 _ptr(g), _ptr(ga), _ptr(gb), _stream(dev))
        return ga.reshape(ctx.shape), gb.reshape(ctx.shape), None, None


def patch_zncc(a, b, mask, *, epsilon=1e-8):
    """``matching.patch_zncc@1``: masked zero-mean normalised cross-correlation of patch
    pairs a, b [..., S] with a 0/1 mask [..., S] -> (correlation [...], valid [...] bool);
    differentiable in a and b (reference.py:225-236).  The mask is not differentiated."""
    _require_cuda_f32("matching.patch_zncc@1", a, b, mask)
    if a.ndim < 1 or a.shape != b.shape or a.shape != mask.shape:
        raise ValueError("patch_zncc: a, b and mask must share one shape [..., S]")
    return _PatchZncc.apply(a, b, mask, float(epsilon))


# ---------------------------------------------------------------- small geometry ops
def pixel_rays(K, *, width, height):
    """``camera.pixel_rays@1``: inv(K) (u + 0.5, v + 0.5, 1) as [height, width, 3]."""
    dev = _require_cuda_f32("camera.pixel_rays@1", K)
    if int(width) <= 0 or int(height) <= 0:
        raise ValueError("pixel_rays: width and height must be positive")
    with torch.cuda.device(dev), torch.no_grad():
        out = torch.empty((int(height), int(width), 3), device=dev, dtype=torch.float32)
        call("sf_b200_pixel_rays", _ptr(K.contiguous()), int(width), int(height), _ptr(out), _stream(dev))
    return out


def ray_peak(means, inverse_covariances, origins, directions):
    """``gaussian.ray_peak@1``: (t [N,P], response [N,P], normals [N,P,3]); forward only."""
    dev = _require_cuda_f32("gaussian.ray_peak@1", means, inverse_covariances, origins, directions)
    with torch.cuda.device(dev), torch.no_grad():
        m, q, o, d = (t.contiguous() for t in (means, inverse_covariances, origins, directions))
        N, P = m.shape[0], o.shape[0]
        t = torch.empty((N, P), device=dev, dtype=torch.float32)
        r = torch.empty((N, P), device=dev, dtype=torch.float32)
        nrm = torch.empty((N, P, 3), device=dev, dtype=torch.float32)
        call("sf_b200_ray_peak", _ptr(m), _ptr(q), N, _ptr(o), _ptr(d), P, _ptr(t), _ptr(r), _ptr(nrm), _stream(dev))
    return t, r, nrm


class _DepthNormals(torch.autograd.Function):
    @staticmethod
    def forward(ctx, depth, K):
        dev = depth.device
        d, k = depth.contiguous(), K.contiguous()
        H, W = d.shape
        normals = torch.empty((H, W, 3), device=dev, dtype=torch.float32)
        valid = torch.empty((H, W), device=dev, dtype=torch.uint8)
        call("sf_b200_depth_normals", _ptr(d), _ptr(k), W, H, _ptr(normals), _ptr(valid), _stream(dev))
        ctx.save_for_backward(d, k)
        ctx.mark_non_differentiable(valid)
        return normals, valid.bool()

    @staticmethod
    def backward(ctx, g_normals, g_valid):
        d, k = ctx.saved_tensors
        dev = d.device
        H, W = d.shape
        if g_normals is None:
            return None, None
        gd = torch.empty_like(d)
        ws = torch.empty((6 * H * W,), device=dev, dtype=torch.float32)
        call("sf_b200_depth_normals_backward", _ptr(d), _ptr(k), W, H, _ptr(g_normals.contiguous()), _ptr(gd), _ptr(ws),
             _stream(dev))
        return gd, None


def depth_normals(depth, K):
    """``geometry.depth_normals@1``: (normals [H,W,3], valid [H,W] bool); differentiable
    with respect to depth (the normal-consistency losses backpropagate through it)."""
    dev = _require_cuda_f32("geometry.depth_normals@1", depth, K)
    with torch.cuda.device(dev):
        return _DepthNormals.apply(depth, K)
