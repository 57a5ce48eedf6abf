"""Tiled renderer restatement (TEST INFRASTRUCTURE; see ``oracle/__init__.py``).

Restates the Torch provider's differentiable renderer:

* projection (src/splatforge/studio/renderers.py:76-107),
* conic / radius / antialiasing (src/splatforge/studio/batched_renderer.py:57-68),
* SH colours and pixel rays (batched_renderer.py:69-83),
* mode extras (batched_renderer.py:90-115),
* exact tile lists (src/splatforge/studio/tile_binning.py:10-34),
* batched, padded per-tile evaluation, compositing and epilogue (batched_renderer.py:127-150, 169-370),
* ``absgrad`` hooks on the projected means (batched_renderer.py:246-280).

Gradients come from autograd through this composition, as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .binning import tile_lists


@dataclass
class RenderSettings:
    """The hot-path fields of ``RenderConfig`` (src/splatforge/studio/config.py:29-40)."""

    tile_size: int = 16
    sigma_extent: float = 3.0
    eps2d: float = 0.3
    near: float = 0.01
    far: float = 10000.0
    background: tuple = (1.0, 1.0, 1.0)
    antialiased: bool = False


CHANNELS = (
    ("rgb", 3),
    ("alpha", 1),
    ("depth", 1),
    ("normals", 3),
    ("distortion_l1", 1),
    ("distortion_l2", 1),
    ("median_depth", 1),
    ("ray_color", 1),
    ("ambiguity_mask", 1),
)


def project(view, camera, eps2d, near):
    """World -> camera, EWA Jacobian with the z <= near guard, screen covariance
    (renderers.py:76-107).

    Every quantity that feeds a discrete decision downstream (depth order, the
    tile rectangle, the ``squared <= extent^2`` mask) is evaluated here as a
    fixed sequence of correctly rounded float32 operations -- sums over the
    inner index in ascending order, no fused multiply-add -- so that the CUDA
    kernels, which perform the same sequence with ``__fmul_rn``/``__fadd_rn``,
    reproduce those decisions bit for bit.  The matrix products are the same
    products the reference writes with ``@``.
    """
    W = camera.world_to_camera
    R, t = W[:3, :3], W[:3, 3]
    mu = view.means
    m = torch.stack(
        [((R[i, 0] * mu[:, 0] + R[i, 1] * mu[:, 1]) + R[i, 2] * mu[:, 2]) + t[i] for i in range(3)], -1
    )
    cov = covariance_explicit(view.quats, view.scales)
    A = [[(R[i, 0] * cov[:, 0, j] + R[i, 1] * cov[:, 1, j]) + R[i, 2] * cov[:, 2, j] for j in range(3)] for i in range(3)]
    cov_cam = torch.stack(
        [torch.stack([(A[i][0] * R[j, 0] + A[i][1] * R[j, 1]) + A[i][2] * R[j, 2] for j in range(3)], -1) for i in range(3)],
        -2,
    )
    x, y, z = m.unbind(-1)
    active = z > near
    zs = torch.where(active, z, torch.ones_like(z))
    x = torch.where(active, x, torch.zeros_like(x))
    y = torch.where(active, y, torch.zeros_like(y))
    zero = torch.zeros_like(z)
    K = camera.K
    fx, fy = K[0, 0], K[1, 1]
    zz = zs * zs
    j00, j02 = fx / zs, (-fx * x) / zz
    j11, j12 = fy / zs, (-fy * y) / zz
    J = torch.stack((j00, zero, j02, zero, j11, j12), -1).reshape(-1, 2, 3)
    xy = torch.stack(((fx * x) / zs + K[0, 2], (fy * y) / zs + K[1, 2]), -1)
    c = cov_cam
    T0 = [j00 * c[:, 0, k] + j02 * c[:, 2, k] for k in range(3)]
    T1 = [j11 * c[:, 1, k] + j12 * c[:, 2, k] for k in range(3)]
    s00 = T0[0] * j00 + T0[2] * j02
    s01 = T0[1] * j11 + T0[2] * j12
    s11 = T1[1] * j11 + T1[2] * j12
    screen = torch.stack((s00, s01, s01, s11), -1).reshape(-1, 2, 2)
    filtered = torch.stack((s00 + eps2d, s01, s01, s11 + eps2d), -1).reshape(-1, 2, 2)
    return m, cov_cam, J, xy, screen, filtered


def _sqrt_rn(x):
    """Correctly rounded float32 square root (torch's vectorised float32 sqrt is not
    always correctly rounded; via float64 it is, since 53 >= 2*24 + 2)."""
    return x.double().sqrt().to(x.dtype) if x.dtype == torch.float32 else x.sqrt()


def rotation_explicit(quats):
    """The rotation of ``rotation_matrix`` (reference.py:15-31) as explicit float32
    operations: ``n = sqrt(((w^2 + x^2) + y^2) + z^2)`` and the reference's formula on
    the normalised quaternion.  Returns nested lists R[i][j] of [N] tensors."""
    w, x, y, z = quats.unbind(-1)
    n = _sqrt_rn(((w * w + x * x) + y * y) + z * z).clamp_min(1e-12)
    w, x, y, z = w / n, x / n, y / n, z / n
    return [
        [1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
        [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
        [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
    ]


def dot3_rn(a, b):
    """``(a0 b0 + a1 b1) + a2 b2`` over the last dimension, each product and sum rounded
    on its own."""
    return (a[..., 0] * b[..., 0] + a[..., 1] * b[..., 1]) + a[..., 2] * b[..., 2]


def ambisur_plane(view, camera, m):
    """AmbiSuR camera-facing normal and plane distance (batched_renderer.py:96-108): the
    rotation column of the smallest scale, turned into the camera frame, flipped to face
    the camera, and its dot product with the camera-space mean, as explicit float32
    sums (the per-pixel plane depth plane / (n . ray) is ill-conditioned at grazing
    angles, so the kernels evaluate the same sequence)."""
    axis = view.scales.detach().argmin(-1)
    R = rotation_explicit(view.quats)
    cols = torch.stack([torch.stack(row, -1) for row in R], -2)  # [N, 3, 3]
    world = cols.gather(2, axis[:, None, None].expand(-1, 3, 1)).squeeze(-1)
    Wc = camera.world_to_camera[:3, :3]
    nc = torch.stack([dot3_rn(world, Wc[i].expand_as(world)) for i in range(3)], -1)
    facing = dot3_rn(nc, m)
    normals = torch.where(facing[:, None] > 0, -nc, nc)
    return normals, dot3_rn(normals, m)


def covariance_explicit(quats, scales):
    """``gaussian.covariance@1`` (reference.py:15-35) as explicit float32 sums: the
    rotation of ``rotation_explicit``, ``M = R diag(s*s)``,
    ``C_ij = (M_i0 R_j0 + M_i1 R_j1) + M_i2 R_j2``."""
    R = rotation_explicit(quats)
    s2 = [scales[:, k] * scales[:, k] for k in range(3)]
    M = [[R[i][k] * s2[k] for k in range(3)] for i in range(3)]
    C = [[(M[i][0] * R[j][0] + M[i][1] * R[j][1]) + M[i][2] * R[j][2] for j in range(3)] for i in range(3)]
    return torch.stack([torch.stack(row, -1) for row in C], -2)


def conic_and_radius(filtered, extent):
    """Explicit 2x2 inverse and largest eigenvalue of the filtered covariance
    (batched_renderer.py:57-59 writes ``linalg.inv`` and ``eigvalsh``)."""
    fa, fb, fc = filtered[:, 0, 0], filtered[:, 0, 1], filtered[:, 1, 1]
    det = fa * fc - fb * fb
    conic = torch.stack((fc / det, -fb / det, -fb / det, fa / det), -1).reshape(-1, 2, 2)
    mid = 0.5 * (fa + fc)
    half = 0.5 * (fa - fc)
    lam = mid + _sqrt_rn(half * half + fb * fb)
    return conic, extent * _sqrt_rn(lam.clamp_min(0))


def pixel_grid(camera, Kinv, top, left, h, w):
    """Rays ``inv(K)(u+.5, v+.5, 1)`` and the pixel coordinates ``K ray`` of one
    tile, as explicit float32 sums (renderers.py:233-234, reference.py:49-56)."""
    dev, dt = camera.K.device, camera.K.dtype
    v, u = torch.meshgrid(
        torch.arange(top, top + h, device=dev, dtype=dt) + 0.5,
        torch.arange(left, left + w, device=dev, dtype=dt) + 0.5,
        indexing="ij",
    )
    u, v = u.reshape(-1), v.reshape(-1)
    Ki, K = Kinv, camera.K
    r = [(u * Ki[i, 0] + v * Ki[i, 1]) + Ki[i, 2] for i in range(3)]
    px = (r[0] * K[0, 0] + r[1] * K[0, 1]) + r[2] * K[0, 2]
    py = (r[0] * K[1, 0] + r[1] * K[1, 1]) + r[2] * K[1, 2]
    return torch.stack(r, -1), torch.stack((px, py), -1)


def mahalanobis2(delta, conic):
    """``delta^T Q delta`` as ``dx (Q delta)_x + dy (Q delta)_y``."""
    dx, dy = delta[..., 0], delta[..., 1]
    qa, qb, qc = conic[..., 0, 0], conic[..., 0, 1], conic[..., 1, 1]
    return dx * (qa * dx + qb * dy) + dy * (qb * dx + qc * dy)


def prepare(
    view,
    camera,
    *,
    mode,
    settings=None,
    selected=None,
    distortions="both",
    trunc_sigma=2.0,
):
    """Everything ``render`` computes before its tile loop (batched_renderer.py:
    169-224): projection, conics, colours, mode extras and the exact tile lists.
    Returns a dict that ``tile_batches`` / ``render_batch`` consume."""
    s = settings or RenderSettings()
    if mode not in ("radegs", "gof", "ambisur"):
        raise ValueError(f"unsupported rendering mode: {mode}")
    m, cov_cam, J, xy, screen, filtered = project(view, camera, s.eps2d, s.near)
    if xy.requires_grad:
        xy.retain_grad()
        xy.absgrad = torch.zeros_like(xy)
    extent = trunc_sigma if mode == "ambisur" else s.sigma_extent
    conic, radii = conic_and_radius(filtered, extent)
    opacity = view.opacities
    if s.antialiased:
        opacity = opacity * (
            torch.linalg.det(screen).clamp_min(0) / torch.linalg.det(filtered).clamp_min(1e-12)
        ).sqrt()
    origin = camera.origin
    colors = ops.sh_color(view.sh, view.means - origin, degree=view.sh_degree)
    ray_colors = ops.sh_color(view.sh, view.means.detach() - origin, degree=view.sh_degree)
    Kinv = torch.linalg.inv(camera.K.cpu()).to(camera.K.device)
    n = len(m)
    normals = m.new_zeros((n, 3))
    gain = m.new_zeros((n, 2))
    qinv = torch.eye(3, device=m.device, dtype=m.dtype).expand(n, 3, 3)
    plane = m.new_zeros(n)
    if mode == "radegs":
        full = torch.cat((J, ops._unit(m)[:, None]), 1)
        Tm = full @ cov_cam @ full.transpose(-1, -2)
        gain = (Tm[:, 2:3, :2] @ torch.linalg.inv(Tm[:, :2, :2])).squeeze(1)
        rn = torch.cat((gain, -torch.ones_like(gain[:, :1])), 1)
        normals = ops._unit((full.transpose(-1, -2) @ rn.unsqueeze(-1)).squeeze(-1))
    elif mode == "ambisur":
        normals, plane = ambisur_plane(view, camera, m)
    else:
        qinv = torch.linalg.inv(cov_cam)
    sel = (
        selected
        if selected is not None
        else torch.zeros(n, dtype=torch.bool, device=m.device)
    )
    bounds = torch.cat((xy.detach(), radii.detach()[:, None], m.detach()[:, 2:3]), 1).cpu().numpy()
    ts = s.tile_size
    offsets, ids_all, _ = tile_lists(
        bounds, width=camera.width, height=camera.height, tile_size=ts, near=s.near, far=s.far
    )
    focal = torch.stack((camera.K[0, 0], camera.K[1, 1]))
    bg = m.new_tensor(s.background)
    return dict(
        camera=camera, Kinv=Kinv, settings=s, mode=mode, extent=extent, distortions=distortions,
        offsets=offsets, ids_all=ids_all, xy=xy, radii=radii, conic=conic, colors=colors,
        ray_colors=ray_colors, opacity=opacity, m=m, normals=normals, gain=gain, qinv=qinv,
        plane=plane, sel=sel, focal=focal, bg=bg,
    )


def tile_batches(ctx, tile_batch_size=64, tile_event_budget=1_048_576):
    """Tile batches as the Torch provider forms them (batched_renderer.py:127-150,
    337-370): tiles grouped, in raster order of first appearance, by (height, width,
    bit length of len-1); each group cut into consecutive batches of at most
    min(tile_batch_size, tile_event_budget // (longest * height * width)) tiles, every
    list padded to the group's longest.  Returns [(tile indices, longest), ...]."""
    camera, ts = ctx["camera"], ctx["settings"].tile_size
    cols = (camera.width + ts - 1) // ts
    rows = (camera.height + ts - 1) // ts
    lens = np.diff(ctx["offsets"])
    groups = {}
    for t in range(rows * cols):
        h = min(ts, camera.height - (t // cols) * ts)
        w = min(ts, camera.width - (t % cols) * ts)
        groups.setdefault((h, w, max(1, int(lens[t] - 1).bit_length())), []).append(t)
    batches = []
    for (h, w, _), members in groups.items():
        longest = max(1, int(max(lens[t] for t in members)))
        size = max(1, min(tile_batch_size, tile_event_budget // (longest * h * w)))
        for i in range(0, len(members), size):
            batches.append((members[i : i + size], longest))
    return batches


def render_batch(ctx, tiles, longest):
    """[B, h*w, 13] channel blocks of a batch of equally sized tiles."""
    camera, s = ctx["camera"], ctx["settings"]
    ts = s.tile_size
    cols = (camera.width + ts - 1) // ts
    offsets, ids_all = ctx["offsets"], ctx["ids_all"]
    idx = np.zeros((len(tiles), longest), np.int64)
    gate = np.zeros((len(tiles), longest), bool)
    trays, pix = [], []
    for row, t in enumerate(tiles):
        lo, hi = offsets[t], offsets[t + 1]
        idx[row, : hi - lo], gate[row, : hi - lo] = ids_all[lo:hi], True
        top, left = (t // cols) * ts, (t % cols) * ts
        h, w = min(ts, camera.height - top), min(ts, camera.width - left)
        r, p = pixel_grid(camera, ctx["Kinv"], top, left, h, w)
        trays.append(r)
        pix.append(p)
    dev = ctx["m"].device
    c = ctx
    return _tile_batch(
        torch.as_tensor(idx, device=dev), torch.as_tensor(gate, device=dev), torch.stack(trays),
        torch.stack(pix), camera, c["xy"], c["conic"], c["colors"], c["ray_colors"], c["opacity"],
        c["m"], c["normals"], c["gain"], c["qinv"], c["plane"], c["sel"], c["focal"], c["bg"],
        c["mode"], c["extent"], s, c["distortions"],
    )


def render(
    view,
    camera,
    *,
    mode,
    settings=None,
    selected=None,
    distortions="both",
    trunc_sigma=2.0,
):
    """Returns a dict of HWC images plus ``projected_means`` / ``projected_radii``."""
    ctx = prepare(view, camera, mode=mode, settings=settings, selected=selected,
                  distortions=distortions, trunc_sigma=trunc_sigma)
    ts = ctx["settings"].tile_size
    cols = (camera.width + ts - 1) // ts
    rows = (camera.height + ts - 1) // ts
    blocks = [None] * (rows * cols)
    for tiles, longest in tile_batches(ctx):
        out = render_batch(ctx, tiles, longest)
        for row, t in enumerate(tiles):
            h = min(ts, camera.height - (t // cols) * ts)
            w = min(ts, camera.width - (t % cols) * ts)
            blocks[t] = out[row].reshape(h, w, -1)
    image = torch.cat([torch.cat(blocks[r * cols : (r + 1) * cols], 1) for r in range(rows)], 0)
    parts = torch.split(image, [c for _, c in CHANNELS], dim=-1)
    result = {name: part for (name, _), part in zip(CHANNELS, parts)}
    result["projected_means"] = ctx["xy"]
    result["projected_radii"] = ctx["radii"]
    result["distortion_profile"] = distortions
    return result


def _tile_batch(ids, valid, trays, pix, camera, xy, conic, colors, ray_colors, opacity, m, normals,
                gain, qinv, plane, sel, focal, bg, mode, extent, s, distortions):
    """A batch of B tiles with padded lists ``ids`` [B, M] (``valid`` marks the real
    entries): [B, M, P] evaluation, compositing and epilogue (batched_renderer.py:
    169-338, the uncompiled path)."""
    delta = pix[:, None] - xy[ids][:, :, None, :]
    sq = mahalanobis2(delta, conic[ids][:, :, None])
    P = trays.shape[1]
    if mode == "gof":
        pxy = (xy[ids] - camera.K[:2, 2]) * m[ids, 2:3] / focal
        proxy = torch.cat((pxy, m[ids, 2:3]), -1)[:, :, None, :].expand(-1, -1, P, -1)
        if proxy.requires_grad:
            zdet = m[ids, 2].detach()

            def hook(g, idx=ids, gt=valid, zz=zdet, target=xy):
                value = (g[..., :2] * zz[:, :, None, None] / focal).abs().sum(2)
                target.absgrad.index_add_(0, idx[gt], value[gt])

            proxy.register_hook(hook)
        qd = torch.einsum("bmij,bpj->bmpi", qinv[ids], trays)
        den = (qd * trays[:, None]).sum(-1).clamp_min(1e-12)
        depth = (proxy * qd).sum(-1) / den
        off = depth[..., None] * trays[:, None] - proxy
        e = torch.einsum("bmpi,bmij,bmpj->bmp", off, qinv[ids], off)
        resp = torch.exp(-0.5 * e.clamp_min(0))
        pn = ops._unit(-qd)
    else:
        if delta.requires_grad:

            def hook(g, idx=ids, gt=valid, target=xy):
                target.absgrad.index_add_(0, idx[gt], g.abs().sum(2)[gt])

            delta.register_hook(hook)
        resp = torch.exp(-0.5 * sq)
        pn = normals[ids][:, :, None, :].expand(-1, -1, P, -1)
        if mode == "radegs":
            depth = (
                torch.linalg.vector_norm(m[ids], dim=-1)[:, :, None]
                + (gain[ids][:, :, None, :] * delta).sum(-1)
            ) / torch.linalg.vector_norm(trays, dim=-1)[:, None]
        else:
            den = dot3_rn(pn, trays[:, None].expand_as(pn))
            ok = den.abs() > 1e-8
            depth = plane[ids][:, :, None] / torch.where(ok, den, torch.ones_like(den))
            resp = torch.where(ok, resp, 0)
    keep = valid[:, :, None] & (sq <= extent**2) & (depth > s.near) & (depth < s.far)
    resp = torch.where(keep, resp, 0)
    rgb, alpha, znum, nnum, l1, l2, median, wts = ops.alpha_composite_batch(
        opacity[ids][:, :, None] * resp, colors[ids], depth, pn, distortions=distortions,
    )
    expected = znum / alpha.clamp_min(1e-8)
    if mode == "ambisur":
        dnum = (wts * plane[ids][:, :, None]).sum(1)
        den = (nnum * trays).sum(-1)
        ok = den.abs() > 1e-8
        expected = torch.where(ok, dnum / torch.where(ok, den, torch.ones_like(den)), 0)
    expected = torch.where(alpha > 1e-8, expected, 0)
    var = (
        ops.ray_color_variance_batch(wts, ray_colors[ids], rgb)
        if mode == "ambisur"
        else torch.zeros_like(alpha)
    )
    amb = (wts * sel[ids][:, :, None].to(wts.dtype)).sum(1)
    return torch.cat(
        (
            rgb + (1 - alpha[..., None]) * bg,
            alpha[..., None],
            expected[..., None],
            ops._unit(nnum),
            l1[..., None],
            l2[..., None],
            median[..., None],
            var[..., None],
            amb[..., None],
        ),
        -1,
    )


def training_profile(mode, geometric=True):
    """``render_training`` distortion selection (batched_renderer.py:37-43)."""
    if mode == "ambisur" or not geometric:
        return "none"
    return "l1" if mode == "gof" else "l2"
