"""Tiled renderer restatement (TEST INFRASTRUCTURE; see ``oracle/__init__.py``).

Restates the Torch provider's differentiable renderer:

* projection (src/splatforge/studio/renderers.py:76-107),
* conic / radius / antialiasing (src/splatforge/studio/batched_renderer.py:57-68),
* SH colours and pixel rays (batched_renderer.py:69-83),
* mode extras (batched_renderer.py:90-115),
* exact tile lists (src/splatforge/studio/tile_binning.py:10-34),
* per-tile evaluation, compositing and epilogue (batched_renderer.py:169-338),
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
    """World -> camera, EWA Jacobian with the z <= near guard, screen covariance."""
    R = camera.world_to_camera[:3, :3]
    m = view.means @ R.T + camera.world_to_camera[:3, 3]
    cov = ops.covariance(view.quats, view.scales)
    cov_cam = R @ cov @ R.T
    x, y, z = m.unbind(-1)
    active = z > near
    zs = torch.where(active, z, torch.ones_like(z))
    x = torch.where(active, x, torch.zeros_like(x))
    y = torch.where(active, y, torch.zeros_like(y))
    zero = torch.zeros_like(z)
    fx, fy = camera.K[0, 0], camera.K[1, 1]
    J = torch.stack(
        (fx / zs, zero, -fx * x / zs.square(), zero, fy / zs, -fy * y / zs.square()), -1
    ).reshape(-1, 2, 3)
    xy = torch.stack((fx * x / zs + camera.K[0, 2], fy * y / zs + camera.K[1, 2]), -1)
    screen = J @ cov_cam @ J.transpose(-1, -2)
    filtered = screen + torch.eye(2, device=m.device, dtype=m.dtype) * eps2d
    return m, cov_cam, J, xy, screen, filtered


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
    s = settings or RenderSettings()
    if mode not in ("radegs", "gof", "ambisur"):
        raise ValueError(f"unsupported rendering mode: {mode}")
    m, cov_cam, J, xy, screen, filtered = project(view, camera, s.eps2d, s.near)
    if xy.requires_grad:
        xy.retain_grad()
        xy.absgrad = torch.zeros_like(xy)
    conic = torch.linalg.inv(filtered)
    extent = trunc_sigma if mode == "ambisur" else s.sigma_extent
    radii = extent * torch.linalg.eigvalsh(filtered)[:, -1].clamp_min(0).sqrt()
    opacity = view.opacities
    if s.antialiased:
        opacity = opacity * (
            torch.linalg.det(screen).clamp_min(0) / torch.linalg.det(filtered).clamp_min(1e-12)
        ).sqrt()
    origin = camera.origin
    colors = ops.sh_color(view.sh, view.means - origin, degree=view.sh_degree)
    ray_colors = ops.sh_color(view.sh, view.means.detach() - origin, degree=view.sh_degree)
    rays = ops.pixel_rays(camera.K, width=camera.width, height=camera.height)
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
        axis = view.scales.detach().argmin(-1)
        world = ops.rotation_matrix(view.quats).gather(2, axis[:, None, None].expand(-1, 3, 1)).squeeze(-1)
        normals = world @ camera.world_to_camera[:3, :3].T
        normals = torch.where((normals * m).sum(-1, keepdim=True) > 0, -normals, normals)
        plane = (normals * m).sum(-1)
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
    cols = (camera.width + ts - 1) // ts
    rows_out = []
    tile_index = 0
    for top in range(0, camera.height, ts):
        row = []
        for left in range(0, camera.width, ts):
            h, w = min(ts, camera.height - top), min(ts, camera.width - left)
            ids = torch.as_tensor(
                ids_all[offsets[tile_index] : offsets[tile_index + 1]], device=m.device
            )
            tile_index += 1
            trays = rays[top : top + h, left : left + w].reshape(-1, 3)
            out = _tile(
                ids, trays, camera, xy, conic, colors, ray_colors, opacity, m, normals,
                gain, qinv, plane, sel, focal, bg, mode, extent, s, distortions,
            )
            row.append(out.reshape(h, w, -1))
        rows_out.append(torch.cat(row, 1))
    image = torch.cat(rows_out, 0)
    parts = torch.split(image, [c for _, c in CHANNELS], dim=-1)
    result = {name: part for (name, _), part in zip(CHANNELS, parts)}
    result["projected_means"] = xy
    result["projected_radii"] = radii
    result["distortion_profile"] = distortions
    return result


def _tile(ids, trays, camera, xy, conic, colors, ray_colors, opacity, m, normals,
          gain, qinv, plane, sel, focal, bg, mode, extent, s, distortions):
    """One tile: [L, P] evaluation, compositing and epilogue (batched_renderer.py:185-338)."""
    pix = (trays @ camera.K.T)[:, :2]
    delta = pix.unsqueeze(0) - xy[ids][:, None, :]
    sq = torch.einsum("lpi,lij,lpj->lp", delta, conic[ids], delta)
    P = trays.shape[0]
    if mode == "gof":
        pxy = (xy[ids] - camera.K[:2, 2]) * m[ids, 2:3] / focal
        proxy = torch.cat((pxy, m[ids, 2:3]), -1)[:, None, :].expand(-1, P, -1)
        if proxy.requires_grad:
            zdet = m[ids, 2].detach()

            def hook(g, idx=ids, zz=zdet, target=xy):
                target.absgrad.index_add_(0, idx, (g[..., :2] * zz[:, None, None] / focal).abs().sum(1))

            proxy.register_hook(hook)
        qd = torch.einsum("lij,pj->lpi", qinv[ids], trays)
        den = (qd * trays[None]).sum(-1).clamp_min(1e-12)
        depth = (proxy * qd).sum(-1) / den
        off = depth[..., None] * trays[None] - proxy
        e = torch.einsum("lpi,lij,lpj->lp", off, qinv[ids], off)
        resp = torch.exp(-0.5 * e.clamp_min(0))
        pn = ops._unit(-qd)
    else:
        if delta.requires_grad:

            def hook(g, idx=ids, target=xy):
                target.absgrad.index_add_(0, idx, g.abs().sum(1))

            delta.register_hook(hook)
        resp = torch.exp(-0.5 * sq)
        pn = normals[ids][:, None, :].expand(-1, P, -1)
        if mode == "radegs":
            depth = (
                torch.linalg.vector_norm(m[ids], dim=-1)[:, None]
                + (gain[ids][:, None, :] * delta).sum(-1)
            ) / torch.linalg.vector_norm(trays, dim=-1)[None]
        else:
            den = (pn * trays[None]).sum(-1)
            ok = den.abs() > 1e-8
            depth = plane[ids][:, None] / torch.where(ok, den, torch.ones_like(den))
            resp = torch.where(ok, resp, 0)
    resp = torch.where((sq <= extent**2) & (depth > s.near) & (depth < s.far), resp, 0)
    rgb, alpha, znum, nnum, l1, l2, median, wts = ops.alpha_composite_batch(
        (opacity[ids][:, None] * resp)[None], colors[ids][None], depth[None], pn[None],
        distortions=distortions,
    )
    rgb, alpha, znum, nnum, l1, l2, median, wts = (t[0] for t in (rgb, alpha, znum, nnum, l1, l2, median, wts))
    expected = znum / alpha.clamp_min(1e-8)
    if mode == "ambisur":
        dnum = (wts * plane[ids][:, None]).sum(0)
        den = (nnum * trays).sum(-1)
        ok = den.abs() > 1e-8
        expected = torch.where(ok, dnum / torch.where(ok, den, torch.ones_like(den)), 0)
    expected = torch.where(alpha > 1e-8, expected, 0)
    var = (
        ops.ray_color_variance(wts, ray_colors[ids], rgb)
        if mode == "ambisur"
        else torch.zeros_like(alpha)
    )
    amb = (wts * sel[ids][:, None].to(wts.dtype)).sum(0)
    return torch.cat(
        (
            rgb + (1 - alpha[:, None]) * bg,
            alpha[:, None],
            expected[:, None],
            ops._unit(nnum),
            l1[:, None],
            l2[:, None],
            median[:, None],
            var[:, None],
            amb[:, None],
        ),
        -1,
    )


def training_profile(mode, geometric=True):
    """``render_training`` distortion selection (batched_renderer.py:37-43)."""
    if mode == "ambisur" or not geometric:
        return "none"
    return "l1" if mode == "gof" else "l2"
