"""Operator-level restatements (TEST INFRASTRUCTURE; see ``oracle/__init__.py``).

Each function restates one versioned operator contract of
``src/splatforge/gaussian/semantics.json`` following the reference provider
``src/splatforge/providers/torch/gaussian/reference.py`` (line numbers cited
per function).  Tensors stay on their device and dtype.
"""

from __future__ import annotations

import math

import torch


def _unit(v, dim=-1, eps=1e-12):
    """``F.normalize``: v / max(||v||, eps)."""
    return v / torch.linalg.vector_norm(v, dim=dim, keepdim=True).clamp_min(eps)


def rotation_matrix(quats):
    """wxyz quaternion -> R, after normalisation (reference.py:15-30)."""
    w, x, y, z = _unit(quats).unbind(-1)
    rows = (
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
    )
    return torch.stack(rows, -1).reshape(*quats.shape[:-1], 3, 3)


def covariance(quats, scales):
    """``gaussian.covariance@1``: R diag(s^2) R^T (reference.py:33-35)."""
    R = rotation_matrix(quats)
    return (R * scales.square().unsqueeze(-2)) @ R.transpose(-1, -2)


def ray_peak(means, inverse_covariances, origins, directions):
    """``gaussian.ray_peak@1`` (reference.py:38-46)."""
    delta = origins.unsqueeze(0) - means.unsqueeze(1)
    qd = torch.einsum("nij,pj->npi", inverse_covariances, directions)
    den = torch.einsum("pi,npi->np", directions, qd).clamp_min(1e-12)
    t = -(delta * qd).sum(-1) / den
    off = delta + t.unsqueeze(-1) * directions.unsqueeze(0)
    e = torch.einsum("npi,nij,npj->np", off, inverse_covariances, off)
    return t, torch.exp(-0.5 * e.clamp_min(0)), _unit(-qd)


def pixel_rays(K, *, width, height):
    """``camera.pixel_rays@1``: inv(K) (u+.5, v+.5, 1) (reference.py:49-56)."""
    v, u = torch.meshgrid(
        torch.arange(height, device=K.device, dtype=K.dtype) + 0.5,
        torch.arange(width, device=K.device, dtype=K.dtype) + 0.5,
        indexing="ij",
    )
    pix = torch.stack((u, v, torch.ones_like(u)), -1)
    return pix @ torch.linalg.inv(K).T


def depth_normals(depth, K):
    """``geometry.depth_normals@1`` (reference.py:59-83): back-project z-depth, face
    normals from centred differences, oriented towards the camera; borders and
    pixels with a non-positive neighbour are invalid (zero normal)."""
    height, width = depth.shape
    points = pixel_rays(K, width=width, height=height) * depth.unsqueeze(-1)
    normals = torch.zeros_like(points)
    valid = torch.zeros_like(depth, dtype=torch.bool)
    if height < 3 or width < 3:
        return normals, valid
    dx = points[1:-1, 2:] - points[1:-1, :-2]
    dy = points[2:, 1:-1] - points[:-2, 1:-1]
    n = _unit(torch.linalg.cross(dy, dx))
    facing = (n * points[1:-1, 1:-1]).sum(-1, keepdim=True)
    n = torch.where(facing > 0, -n, n)
    good = (
        (depth[1:-1, 1:-1] > 0) & (depth[1:-1, 2:] > 0) & (depth[1:-1, :-2] > 0)
        & (depth[2:, 1:-1] > 0) & (depth[:-2, 1:-1] > 0)
        & torch.isfinite(n).all(-1) & (n.square().sum(-1) > 0)
    )
    inner = torch.where(good.unsqueeze(-1), n, 0)
    normals = torch.nn.functional.pad(inner.permute(2, 0, 1), (1, 1, 1, 1)).permute(1, 2, 0)
    valid = torch.nn.functional.pad(good, (1, 1, 1, 1))
    return normals, valid


# Real SH basis constants of the gsplat/3DGS convention (reference.py:85-109).
_C0 = 1 / math.sqrt(4 * math.pi)
_C1 = math.sqrt(3 / (4 * math.pi))
_C2 = math.sqrt(15 / (4 * math.pi))
_C2b = math.sqrt(5 / (16 * math.pi))
_C2c = math.sqrt(15 / (16 * math.pi))
_C3 = (
    math.sqrt(35 / (32 * math.pi)),
    math.sqrt(105 / (4 * math.pi)),
    math.sqrt(21 / (32 * math.pi)),
    math.sqrt(7 / (16 * math.pi)),
    math.sqrt(105 / (16 * math.pi)),
)


def sh_basis(x, y, z, degree):
    b = [torch.full_like(x, _C0)]
    if degree >= 1:
        b += [-_C1 * y, _C1 * z, -_C1 * x]
    if degree >= 2:
        b += [
            _C2 * x * y,
            -_C2 * y * z,
            _C2b * (3 * z * z - 1),
            -_C2 * x * z,
            _C2c * (x * x - y * y),
        ]
    if degree >= 3:
        b += [
            -_C3[0] * y * (3 * x * x - y * y),
            _C3[1] * x * y * z,
            -_C3[2] * y * (5 * z * z - 1),
            _C3[3] * z * (5 * z * z - 3),
            -_C3[2] * x * (5 * z * z - 1),
            _C3[4] * z * (x * x - y * y),
            -_C3[0] * x * (x * x - 3 * y * y),
        ]
    return b


def sh_color(coefficients, directions, *, degree):
    """``gaussian.sh_color@1``: max(0, 0.5 + sum_k c_k Y_k(dir)) (reference.py:85-113)."""
    x, y, z = _unit(directions).unbind(-1)
    basis = sh_basis(x, y, z, degree)
    stacked = torch.stack(basis, -1).unsqueeze(-1)
    return (0.5 + (coefficients[:, : len(basis)] * stacked).sum(1)).clamp_min(0)


def sh_ambiguity(coefficients):
    """``gaussian.sh_ambiguity@1`` (reference.py:116-117)."""
    return coefficients[:, 1:].square().sum((1, 2))


def ray_color_variance(weights, colors, composite):
    """``gaussian.ray_color_variance@1`` (reference.py:120-122)."""
    err = colors.unsqueeze(1) - composite.detach().unsqueeze(0)
    return (weights.detach() * err.square().sum(-1)).sum(0)


def ray_color_variance_batch(weights, colors, composite):
    """``gaussian.ray_color_variance@2`` (reference.py:189-191)."""
    err = colors[:, :, None] - composite.detach()[:, None]
    return (weights.detach() * err.square().sum(-1)).sum(1)


def alpha_composite_batch(alphas, colors, depths, normals, *, distortions="both"):
    """``splat.alpha_composite@2/@3`` over [B, N, P] (reference.py:151-186).

    Front-to-back weights w_i = a_i prod_{j<i}(1 - a_j) with a clamped to
    [0, 0.999]; L1 over samples sorted by depth with live weights; L2 with
    detached weights; median = depth at the first cumulative weight >= 0.5.
    """
    a = alphas.clamp(0, 0.999)
    T = torch.cat((torch.ones_like(a[:, :1]), 1 - a), 1).cumprod(1)
    w = a * T[:, :-1]
    alpha = w.sum(1)
    rgb = torch.einsum("bnp,bnc->bpc", w, colors)
    znum = (w * depths).sum(1)
    nnum = (w.unsqueeze(-1) * normals).sum(1)
    wd = w.detach()
    l1 = torch.zeros_like(alpha)
    if distortions in ("l1", "both"):
        sd, order = depths.sort(1)
        sw = w.gather(1, order)
        before_w = sw.cumsum(1) - sw
        before_wd = (sw * sd).cumsum(1) - sw * sd
        l1 = (2 * sw * (sd * before_w - before_wd)).sum(1).clamp_min(0)
    l2 = torch.zeros_like(alpha)
    if distortions in ("l2", "both"):
        l2 = (
            2 * (wd.sum(1) * (wd * depths.square()).sum(1) - (wd * depths).sum(1).square())
        ).clamp_min(0)
    if depths.shape[1]:
        crossed = w.cumsum(1) >= 0.5
        first = crossed.to(torch.int64).argmax(1, keepdim=True)
        median = torch.where(crossed.any(1), depths.gather(1, first).squeeze(1), 0)
    else:
        median = torch.zeros_like(alpha)
    return rgb, alpha, znum, nnum, l1, l2, median, w


def alpha_composite(alphas, colors, depths, normals):
    """``splat.alpha_composite@1``: the unbatched [N, P] form (reference.py:125-148)."""
    out = alpha_composite_batch(
        alphas[None], colors[None], depths[None], normals[None], distortions="both"
    )
    return tuple(t[0] for t in out)


def opacity_field(points, means, inverse_covariances, opacities, origins, *, gaussian_chunk=1024):
    """``gaussian.opacity_field@1`` (reference.py:194-222).

    For every view origin: evaluate each Gaussian along the normalised point ray
    at min(peak t, point distance), drop peaks behind the origin, clamp to
    [0, 0.999], O_view = 1 - prod(1 - c); the field is the minimum over views.
    """
    out = torch.ones(points.shape[0], device=points.device, dtype=points.dtype)
    for o in origins:
        delta = points - o
        dist = torch.linalg.vector_norm(delta, dim=-1)
        dirs = _unit(delta)
        trans = torch.ones_like(out)
        for s in range(0, means.shape[0], gaussian_chunk):
            m = means[s : s + gaussian_chunk]
            q = inverse_covariances[s : s + gaussian_chunk]
            t, _, _ = ray_peak(m, q, o.expand_as(points), dirs)
            te = torch.minimum(t, dist.unsqueeze(0))
            off = o - m.unsqueeze(1) + te.unsqueeze(-1) * dirs
            e = torch.einsum("npi,nij,npj->np", off, q, off)
            c = opacities[s : s + gaussian_chunk, None] * torch.exp(-0.5 * e.clamp_min(0))
            c = torch.where(t > 0, c, 0).clamp(0, 0.999)
            trans = trans * (1 - c).prod(0)
        out = torch.minimum(out, 1 - trans)
    return out


def patch_zncc(a, b, mask, epsilon=1e-8):
    """``matching.patch_zncc@1`` (reference.py:225-236): masked, zero-mean correlation of
    patch pairs over the last axis; a patch needs >= 2 valid samples and both variances
    above epsilon, else it reads 0 and is invalid.  Returns (correlation, valid)."""
    n = mask.sum(-1)
    count = n.clamp_min(1)
    ca = a - (a * mask).sum(-1, keepdim=True) / count[..., None]
    cb = b - (b * mask).sum(-1, keepdim=True) / count[..., None]
    va = (mask * ca * ca).sum(-1)
    vb = (mask * cb * cb).sum(-1)
    ok = (n >= 2) & (va > epsilon) & (vb > epsilon)
    r = (mask * ca * cb).sum(-1) / torch.sqrt((va * vb).clamp_min(epsilon * epsilon))
    return torch.where(ok, r.clamp(-1, 1), torch.zeros_like(r)), ok


def normal_consistency(depth, K, alpha, vector, mask, numerator=True):
    """The normal-consistency loss (studio/losses.py:45-53) on [H,W] depth/alpha/mask and
    an [H,W,3] normal numerator (term alpha - v . n) or unit normals (term 1 - v . n):
    the mean of the term over pixels whose depth normal n is valid, alpha > 0.1 and
    mask > 0 (losses.py:9-12), divided by max(count, 1)."""
    n, valid = depth_normals(depth, K)
    keep = valid & (alpha > 0.1) & (mask > 0)
    dot = (vector * n).sum(-1)
    term = (alpha - dot) if numerator else (1 - dot)
    return torch.where(keep, term, torch.zeros_like(term)).sum() / keep.sum().clamp_min(1)


def densify_observe(gradient, observations, grad2d, radii, scale=(1.0, 1.0)):
    """GaussianDensifier.observe's update (studio/densification.py:18-43): where the
    projected radius is positive, add the norm of the scaled 2D gradient and count one
    observation.  Updates the accumulators in place."""
    seen = radii.reshape(-1) > 0
    g = grad2d.reshape(-1, 2) * grad2d.new_tensor(scale)
    gradient += torch.where(seen, torch.linalg.vector_norm(g, dim=-1), torch.zeros_like(gradient))
    observations += seen.to(observations.dtype)


def sh_ambiguity(coefficients):
    """``gaussian.sh_ambiguity@1`` (reference.py:116-117): squared norm outside the DC band."""
    return (coefficients[:, 1:] * coefficients[:, 1:]).sum((1, 2))


def ray_color_variance_batch(weights, colors, composite):
    """``gaussian.ray_color_variance@2`` (reference.py:189-191): per batch and pixel,
    sum_n stopgrad(w) |c_n - stopgrad(composite)|^2."""
    diff = colors[:, :, None, :] - composite.detach()[:, None, :, :]
    return (weights.detach() * (diff * diff).sum(-1)).sum(1)
