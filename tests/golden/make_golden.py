"""Generate golden fixtures by running SplatForge's own Torch provider.

Run where the reference source tree is present, giving its ``src`` directory as the
first argument or in ``SPLATFORGE_SRC``:

    python tests/golden/make_golden.py <reference>/src [fixture ...]

It imports the reference read-only (no files are written into it), evaluates
its renderers, operators and tile binning on seeded synthetic inputs, and
writes compressed ``.npz`` fixtures next to this script.  The fixtures pin the
CPU oracle (``oracle/``) in ``tests/test_oracle_golden.py``; GPU parity tests
then compare the CUDA path against that pinned oracle.

Fixtures (all float32 unless noted):

* ``binning.npz``   -- the reference's rng(703) tangency fixture plus larger
                       random cases: bounds in, CSR tile lists out (int64).
* ``geometry.npz``  -- pixel_rays@1, ray_peak@1, depth_normals@1 (with the depth
                       adjoint of a seeded loss on the normals).
* ``mesh.npz``      -- marching_tetrahedra on an analytic plane (the reference's own
                       test case) and sphere, and the GOF exporter's gaussian_grid
                       (with and without max_gaussians) plus the level set of the
                       opacity field of a 300-Gaussian scene (float64 grid).
* ``ops_extra.npz`` -- gaussian.sh_ambiguity@1, gaussian.ray_color_variance@1/@2 and
                       splat.alpha_composite@1 with the adjoints of seeded linear losses.
* ``training.npz``  -- matching.patch_zncc@1 (with its a/b adjoints), the
                       normal-consistency loss (numerator and unit-normal forms, with
                       input gradients) and GaussianDensifier.observe statistics.
* ``ops.npz``       -- covariance@1, sh_color@1 (deg 0..3), pixel_rays@1,
                       ray_peak@1, alpha_composite@3 (all profiles, with input
                       gradients), opacity_field@1.
* ``render_<mode>.npz`` -- ``TorchRenderer`` on the 48-Gaussian demo scene, three
                       24x24 views: every image channel, projected means and
                       radii, and the parameter gradients of a seeded linear loss
                       over every channel, plus ``projected_means.grad/.absgrad``.
* ``train_<mode>.npz``  -- ``BatchedTorchRenderer.render_training`` on the same
                       scene (the per-mode distortion profile).
* ``crop_<mode>.npz``   -- ``BatchedTorchRenderer`` on a 48x32 tile-aligned crop of
                       a 20k-Gaussian surface scene (gradients stored sparsely).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _setup(src):
    sys.path.insert(0, str(src))
    sys.path.insert(0, str(REPO))
    sys.dont_write_bytecode = True
    torch.set_num_threads(1)


def binning_cases():
    from splatforge.studio.tile_binning import tile_members

    out = {}
    rng = np.random.default_rng(703)
    b = rng.normal(size=(250, 4)).astype(np.float32)
    b[:, :2] = b[:, :2] * 35 + 16
    b[:, 2] = rng.uniform(0, 45, len(b))
    b[:, 3] = rng.uniform(-1, 10, len(b))
    b[0] = [16, 16, 0, 2]
    b[1] = [40, 24, 7, 2]
    cases = [("fixture703", b, 33, 21, 0.01, 9.0)]
    rng = np.random.default_rng(11)
    for k, (n, w, h) in enumerate(((4000, 200, 150), (3000, 97, 61))):
        bb = np.empty((n, 4), np.float32)
        bb[:, 0] = rng.uniform(-40, w + 40, n)
        bb[:, 1] = rng.uniform(-40, h + 40, n)
        bb[:, 2] = rng.exponential(8.0, n)
        bb[:, 3] = rng.choice(np.linspace(-0.5, 12.0, 300), n)  # many exact depth ties
        bb[:8, :] = [[16, 16, 0, 2], [32, 0, 16, 1], [0, 32, 16, 1], [w, h, 0, 1],
                     [w + 1, h, 1, 1], [-1, -1, 1, 1], [48, 48, 16, 0.01], [48, 48, 16, 12.0]]
        cases.append((f"random{k}", bb, w, h, 0.01, 10.0))
    for name, bounds, w, h, near, far in cases:
        members = tile_members(bounds, width=w, height=h, tile_size=16, near=near, far=far)
        offsets = np.concatenate(([0], np.cumsum([len(m) for m in members]))).astype(np.int64)
        ids = np.concatenate(members).astype(np.int64) if len(members) else np.zeros(0, np.int64)
        out[f"{name}/bounds"] = bounds
        out[f"{name}/meta"] = np.array([w, h, 16, near, far], np.float64)
        out[f"{name}/offsets"] = offsets
        out[f"{name}/ids"] = ids
    np.savez_compressed(HERE / "binning.npz", **out)


def op_cases():
    from splatforge.gaussian import SurfaceOperators

    ops = SurfaceOperators()
    out = {}
    g = torch.Generator().manual_seed(5)
    q = torch.randn(64, 4, generator=g)
    s = torch.rand(64, 3, generator=g) * 0.5 + 0.05
    out["cov/quats"], out["cov/scales"] = q.numpy(), s.numpy()
    out["cov/out"] = ops("gaussian.covariance@1", q, s).numpy()
    sh = torch.randn(64, 16, 3, generator=g) * 0.3
    d = torch.randn(64, 3, generator=g)
    out["sh/coeffs"], out["sh/dirs"] = sh.numpy(), d.numpy()
    for deg in range(4):
        shv = sh.clone().requires_grad_()
        dv = d.clone().requires_grad_()
        col = ops("gaussian.sh_color@1", shv, dv, degree=deg)
        up = torch.randn(col.shape, generator=g)
        gs, gd = torch.autograd.grad((col * up).sum(), (shv, dv), allow_unused=True)
        gd = torch.zeros_like(dv) if gd is None else gd
        out[f"sh/deg{deg}/out"] = col.detach().numpy()
        out[f"sh/deg{deg}/up"] = up.numpy()
        out[f"sh/deg{deg}/gcoeffs"] = gs.numpy()
        out[f"sh/deg{deg}/gdirs"] = gd.numpy()
    K = torch.tensor([[30.0, 0, 17.0], [0, 28.0, 11.0], [0, 0, 1]])
    out["rays/K"] = K.numpy()
    out["rays/out"] = ops("camera.pixel_rays@1", K, width=33, height=21).numpy()
    # ray peak
    m = torch.randn(7, 3, generator=g)
    A = torch.randn(7, 3, 3, generator=g)
    Q = A @ A.transpose(-1, -2) + torch.eye(3)
    o = torch.randn(5, 3, generator=g)
    dd = torch.randn(5, 3, generator=g)
    t, r, n = ops("gaussian.ray_peak@1", m, Q, o, dd)
    out.update({"peak/means": m.numpy(), "peak/Q": Q.numpy(), "peak/o": o.numpy(),
                "peak/d": dd.numpy(), "peak/t": t.numpy(), "peak/r": r.numpy(), "peak/n": n.numpy()})
    # composite @3, every profile, with adjoints
    B, N, P = 3, 9, 11
    a0 = torch.rand(B, N, P, generator=g) * 0.6
    a0[0, 2, :4] = 0.9995  # clamp at 0.999
    a0[1, 3, :3] = -0.01  # clamp at 0
    c0 = torch.rand(B, N, 3, generator=g)
    d0 = torch.rand(B, N, P, generator=g) * 4 + 1
    n0 = torch.randn(B, N, P, 3, generator=g)
    out.update({"comp/a": a0.numpy(), "comp/c": c0.numpy(), "comp/d": d0.numpy(), "comp/n": n0.numpy()})
    ups = None
    for prof in ("none", "l1", "l2", "both"):
        ins = [t.clone().requires_grad_() for t in (a0, c0, d0, n0)]
        res = ops("splat.alpha_composite@3", *ins, distortions=prof)
        if ups is None:
            ups = [torch.randn(r.shape, generator=g) for r in res]
            for i, u in enumerate(ups):
                out[f"comp/up{i}"] = u.numpy()
        loss = sum((r * u).sum() for r, u in zip(res, ups))
        grads = torch.autograd.grad(loss, ins)
        for i, r in enumerate(res):
            out[f"comp/{prof}/out{i}"] = r.detach().numpy()
        for name, gr in zip("acdn", grads):
            out[f"comp/{prof}/g{name}"] = gr.numpy()
    # opacity field
    pts = torch.randn(40, 3, generator=g) * 0.6
    mm = torch.randn(25, 3, generator=g) * 0.5
    L = torch.randn(25, 3, 3, generator=g) * 0.1
    C = L @ L.transpose(-1, -2) + 0.01 * torch.eye(3)
    Qf = torch.linalg.inv(C)
    op = torch.rand(25, generator=g)
    origins = torch.randn(3, 3, generator=g) * 3
    field = ops("gaussian.opacity_field@1", pts, mm, Qf, op, origins)
    out.update({"field/p": pts.numpy(), "field/m": mm.numpy(), "field/Q": Qf.numpy(),
                "field/o": op.numpy(), "field/origins": origins.numpy(), "field/out": field.numpy()})
    np.savez_compressed(HERE / "ops.npz", **out)


def geometry_cases():
    """camera.pixel_rays@1, gaussian.ray_peak@1 and geometry.depth_normals@1 (with the
    depth adjoint of a seeded linear loss on the normals)."""
    from splatforge.gaussian import SurfaceOperators

    ops = SurfaceOperators()
    out = {}
    g = torch.Generator().manual_seed(13)
    K = torch.tensor([[420.0, 0.0, 311.5], [0.0, 415.0, 237.25], [0.0, 0.0, 1.0]])
    out["rays/K"] = K.numpy()
    out["rays/out"] = ops("camera.pixel_rays@1", K, width=64, height=48).numpy()
    m = torch.randn(31, 3, generator=g)
    A = torch.randn(31, 3, 3, generator=g)
    Q = A @ A.transpose(-1, -2) + 0.1 * torch.eye(3)
    o = torch.randn(23, 3, generator=g) * 2
    d = torch.randn(23, 3, generator=g)
    t, r, n = ops("gaussian.ray_peak@1", m, Q, o, d)
    out.update({"peak/means": m.numpy(), "peak/Q": Q.numpy(), "peak/o": o.numpy(), "peak/d": d.numpy(),
                "peak/t": t.numpy(), "peak/r": r.numpy(), "peak/n": n.numpy()})
    H, W = 37, 53
    yy, xx = torch.meshgrid(torch.arange(H, dtype=torch.float32), torch.arange(W, dtype=torch.float32), indexing="ij")
    depth = 2.0 + 0.3 * torch.sin(xx / 7.0) + 0.2 * torch.cos(yy / 5.0) + 0.05 * torch.rand(H, W, generator=g)
    depth[5, 9] = 0.0     # a hole: its neighbours become invalid
    depth[20, 30] = -1.0  # a negative depth
    depth = depth.requires_grad_()
    Kd = torch.tensor([[60.0, 0.0, 26.0], [0.0, 58.0, 18.5], [0.0, 0.0, 1.0]])
    normals, valid = ops("geometry.depth_normals@1", depth, Kd)
    up = torch.randn(normals.shape, generator=g)
    (gd,) = torch.autograd.grad((normals * up).sum(), depth)
    out.update({"dn/depth": depth.detach().numpy(), "dn/K": Kd.numpy(), "dn/normals": normals.detach().numpy(),
                "dn/valid": valid.numpy(), "dn/up": up.numpy(), "dn/gdepth": gd.numpy()})
    np.savez_compressed(HERE / "geometry.npz", **out)


def mesh_cases():
    """marching_tetrahedra on analytic fields, and the GOF exporter's extraction
    (gaussian_grid, opacity_field@1 at every grid and bisection point,
    marching_tetrahedra) of a 300-Gaussian surface scene seen from 4 origins."""
    from types import SimpleNamespace

    from splatforge.gaussian import SurfaceOperators
    from splatforge.mesh.tetrahedra import marching_tetrahedra, triangulate
    from splatforge.studio.exporters import gaussian_grid
    from splatforge_b200 import scenes

    out = {}
    # the reference's analytic-plane case (tests/integration/test_surface_studio.py:108-128)
    cube = np.asarray([[x, y, z] for x in (-1.0, 1.0) for y in (-1.0, 1.0) for z in (-1.0, 1.0)])

    def plane(p):
        return p[:, 2] - 0.25

    cells = triangulate(cube)
    v, f = marching_tetrahedra(cube, cells, plane(cube), plane, binary_steps=12, inside_greater=False)
    out.update({"plane/points": cube, "plane/cells": cells, "plane/vertices": v, "plane/faces": f})

    # a sphere level set over a radius-filtered Delaunay grid of seeded points
    rng = np.random.default_rng(5)
    pts = rng.uniform(-1.0, 1.0, (400, 3))
    radii = rng.uniform(0.3, 0.6, 400)

    def sphere(p):
        return np.sqrt((p * p).sum(-1)) - 0.55

    cells = triangulate(pts, radii)
    v, f = marching_tetrahedra(pts, cells, sphere(pts), sphere, level=0.0, binary_steps=8, inside_greater=False)
    out.update({"sphere/points": pts, "sphere/radii": radii, "sphere/cells": cells, "sphere/vertices": v,
                "sphere/faces": f})

    # GOF extraction
    params = scenes.surfaces(300, seed=4)
    view = scenes.activated(params)
    model = SimpleNamespace(means=view.means, quats=view.quats, scales=view.scales, opacities=view.opacities,
                            device=torch.device("cpu"))
    ops = SurfaceOperators()
    inverse = torch.linalg.inv(ops("gaussian.covariance@1", view.quats, view.scales))
    g = torch.Generator().manual_seed(17)
    d = torch.randn(4, 3, generator=g)
    origins = 3.0 * d / d.norm(dim=-1, keepdim=True)

    def field(coordinates):
        sample = torch.as_tensor(coordinates, dtype=torch.float32)
        return ops("gaussian.opacity_field@1", sample, view.means, inverse, view.opacities, origins,
                   gaussian_chunk=512).numpy()

    for tag, cap in (("gof", None), ("gof_cap", 120)):
        config = SimpleNamespace(seed_opacity_min=0.05, max_gaussians=cap, tetra_extent=3.0)
        points, cells, seeds = gaussian_grid(model, config)
        out.update({f"{tag}/points": points, f"{tag}/cells": cells, f"{tag}/seeds": np.int64(seeds)})
    points, cells = out["gof/points"], out["gof/cells"]
    values = field(points)
    v, f = marching_tetrahedra(points, cells, values, field, level=0.5, binary_steps=8, inside_greater=True)
    out.update({"gof/means": view.means.numpy(), "gof/quats": view.quats.numpy(), "gof/scales": view.scales.numpy(),
                "gof/opacities": view.opacities.numpy(), "gof/inverse": inverse.numpy(),
                "gof/origins": origins.numpy(), "gof/values": values, "gof/vertices": v, "gof/faces": f})
    np.savez_compressed(HERE / "mesh.npz", **out)


def extra_op_cases():
    """gaussian.sh_ambiguity@1 and gaussian.ray_color_variance@1/@2 with the adjoints of
    seeded linear losses."""
    from splatforge.gaussian import SurfaceOperators

    ops = SurfaceOperators()
    g = torch.Generator().manual_seed(31)
    out = {}
    sh = torch.randn(57, 16, 3, generator=g).requires_grad_()
    amb = ops("gaussian.sh_ambiguity@1", sh)
    up = torch.randn(57, generator=g)
    (gsh,) = torch.autograd.grad((amb * up).sum(), sh)
    out.update({"amb/sh": sh.detach().numpy(), "amb/out": amb.detach().numpy(), "amb/up": up.numpy(),
                "amb/gsh": gsh.numpy()})
    B, N, P = 3, 37, 256
    w = torch.rand(B, N, P, generator=g) * 0.1
    c = torch.rand(B, N, 3, generator=g).requires_grad_()
    r = torch.rand(B, P, 3, generator=g)
    var = ops("gaussian.ray_color_variance@2", w, c, r)
    upv = torch.randn(B, P, generator=g)
    (gc,) = torch.autograd.grad((var * upv).sum(), c)
    c1 = c.detach()[0].clone().requires_grad_()
    var1 = ops("gaussian.ray_color_variance@1", w[0], c1, r[0])
    (gc1,) = torch.autograd.grad((var1 * upv[0]).sum(), c1)
    out.update({"rcv/w": w.numpy(), "rcv/c": c.detach().numpy(), "rcv/r": r.numpy(), "rcv/out": var.detach().numpy(),
                "rcv/up": upv.numpy(), "rcv/gc": gc.numpy(), "rcv/out1": var1.detach().numpy(),
                "rcv/gc1": gc1.numpy()})
    # splat.alpha_composite@1 (TorchRenderer's unbatched composite) with input gradients
    N, P = 23, 64
    al = (torch.rand(N, P, generator=g) * 0.9).requires_grad_()
    col = torch.rand(N, 3, generator=g).requires_grad_()
    dep = (1 + torch.rand(N, P, generator=g) * 3).requires_grad_()
    nrm = torch.randn(N, P, 3, generator=g).requires_grad_()
    res = ops("splat.alpha_composite@1", al, col, dep, nrm)
    ups = [torch.randn(r.shape, generator=g) for r in res]
    grads = torch.autograd.grad(sum((r * u).sum() for r, u in zip(res, ups)), (al, col, dep, nrm))
    out.update({"c1/a": al.detach().numpy(), "c1/c": col.detach().numpy(), "c1/d": dep.detach().numpy(),
                "c1/n": nrm.detach().numpy()})
    out.update({f"c1/out{i}": r.detach().numpy() for i, r in enumerate(res)})
    out.update({f"c1/up{i}": u.numpy() for i, u in enumerate(ups)})
    out.update({f"c1/g{k}": gr.numpy() for k, gr in zip("acdn", grads)})
    np.savez_compressed(HERE / "ops_extra.npz", **out)


def training_cases():
    """matching.patch_zncc@1 (forward and the a/b adjoints of a seeded linear loss, with
    short, constant, perfectly correlated and anti-correlated patches), the
    normal-consistency loss with and without a normal numerator (value and input
    gradients), and GaussianDensifier.observe in pixel and NDC gradient space."""
    from types import SimpleNamespace

    from splatforge.gaussian import SurfaceOperators
    from splatforge.studio.densification import GaussianDensifier
    from splatforge.studio.losses import normal_consistency

    ops = SurfaceOperators()
    out = {}
    g = torch.Generator().manual_seed(23)
    rows, S = 40, 49
    a = torch.rand(rows, S, generator=g)
    b = 0.6 * a + 0.4 * torch.rand(rows, S, generator=g)
    m = (torch.rand(rows, S, generator=g) > 0.2).float()
    m[0] = 0.0
    m[1, 1:] = 0.0           # one sample: invalid
    a[2] = 0.5               # constant: zero variance
    b[3] = 2.0 * a[3] + 1.0  # perfectly correlated
    b[4] = -a[4]             # anti-correlated
    a.requires_grad_()
    b.requires_grad_()
    corr, valid = ops("matching.patch_zncc@1", a, b, m)
    up = torch.randn(rows, generator=g)
    ga, gb = torch.autograd.grad((corr * up).sum(), (a, b))
    out.update({"zncc/a": a.detach().numpy(), "zncc/b": b.detach().numpy(), "zncc/m": m.numpy(),
                "zncc/corr": corr.detach().numpy(), "zncc/valid": valid.numpy(), "zncc/up": up.numpy(),
                "zncc/ga": ga.numpy(), "zncc/gb": gb.numpy()})

    H, W = 29, 41
    yy, xx = torch.meshgrid(torch.arange(H, dtype=torch.float32), torch.arange(W, dtype=torch.float32), indexing="ij")
    depth = 2.0 + 0.3 * torch.sin(xx / 6.0) + 0.2 * torch.cos(yy / 4.0) + 0.05 * torch.rand(H, W, generator=g)
    depth[7, 11] = 0.0
    alpha = torch.rand(H, W, generator=g)
    nnum = torch.randn(H, W, 3, generator=g) * 0.5
    normals = torch.nn.functional.normalize(torch.randn(H, W, 3, generator=g), dim=-1)
    mask = (torch.rand(H, W, generator=g) > 0.1).float()
    K = torch.tensor([[50.0, 0.0, 20.0], [0.0, 48.0, 14.5], [0.0, 0.0, 1.0]])
    camera = SimpleNamespace(K=K)
    out.update({"nc/depth": depth.numpy(), "nc/alpha": alpha.numpy(), "nc/nnum": nnum.numpy(),
                "nc/normals": normals.numpy(), "nc/mask": mask.numpy(), "nc/K": K.numpy()})
    for tag, numerator in (("num", True), ("unit", False)):
        d = depth.clone().unsqueeze(-1).requires_grad_()
        al = alpha.clone().unsqueeze(-1).requires_grad_()
        v = (nnum if numerator else normals).clone().requires_grad_()
        output = SimpleNamespace(depth=d, alpha=al, normals=v if not numerator else normals,
                                 normal_numerator=v if numerator else None)
        loss = normal_consistency(output, camera, ops, mask.unsqueeze(-1))
        gd, gal, gv = torch.autograd.grad(loss, (d, al, v), allow_unused=True)
        gal = torch.zeros_like(al) if gal is None else gal
        out.update({f"nc/{tag}/loss": loss.detach().numpy(), f"nc/{tag}/gdepth": gd.squeeze(-1).numpy(),
                    f"nc/{tag}/galpha": gal.squeeze(-1).numpy(), f"nc/{tag}/gvec": gv.numpy()})

    n = 500
    grad = torch.randn(n, 2, generator=g)
    absgrad = grad.abs() + torch.rand(n, 2, generator=g)
    radii = torch.where(torch.rand(n, generator=g) > 0.3, torch.rand(n, generator=g) * 10, torch.zeros(n))
    out.update({"dens/grad": grad.numpy(), "dens/absgrad": absgrad.numpy(), "dens/radii": radii.numpy()})
    for space in ("pixel", "ndc"):
        for absolute in (False, True):
            config = SimpleNamespace(absolute_gradients=absolute, gradient_space=space)
            model = SimpleNamespace(count=n, device=torch.device("cpu"))
            dens = GaussianDensifier(config, model)
            projected = torch.zeros(n, 2)
            projected.grad = grad
            projected.absgrad = absgrad
            output = SimpleNamespace(projected_means=projected, projected_radii=radii, rgb=torch.zeros(24, 40, 3))
            dens.observe(output, model)
            dens.observe(output, model)
            key = f"dens/{space}/{'abs' if absolute else 'grad'}"
            out.update({f"{key}/gradient": dens.gradient.numpy(), f"{key}/observations": dens.observations.numpy()})
    np.savez_compressed(HERE / "training.npz", **out)


CHANNELS = ("rgb", "alpha", "depth", "normals", "distortion_l1", "distortion_l2",
            "median_depth", "ray_color", "ambiguity_mask")


def _view_from(params, GaussianView):
    return GaussianView(params.means, params.quats, params.log_scales.exp(),
                        params.opacity_logits.sigmoid(), params.sh, params.sh_degree)


def _camera(cam, Camera):
    return Camera(cam.K, cam.world_to_camera, cam.width, cam.height, cam.name)


def _run(renderer_call, params, cams, Camera, GaussianView, seed, sparse=False):
    out = {}
    for v, cam in enumerate(cams):
        p = params.detach_clone().requires_grad_()
        view = _view_from(p, GaussianView)
        n = p.means.shape[0]
        selected = torch.arange(n) % 2 == 0
        res = renderer_call(view, _camera(cam, Camera), selected)
        g = torch.Generator().manual_seed(seed + v)
        loss = 0
        for ch in CHANNELS:
            img = getattr(res, ch)
            up = torch.randn(img.shape, generator=g)
            out[f"v{v}/up_{ch}"] = up.numpy()
            out[f"v{v}/{ch}"] = img.detach().numpy()
            loss = loss + (img * up).sum()
        names = ("means", "log_scales", "quats", "opacity_logits", "sh")
        grads = torch.autograd.grad(loss, list(p.tensors()))
        pm = res.projected_means
        # projected_means carries .grad via retain_grad and .absgrad via hooks
        loss2 = 0
        p2 = params.detach_clone().requires_grad_()
        res2 = renderer_call(_view_from(p2, GaussianView), _camera(cam, Camera), selected)
        g = torch.Generator().manual_seed(seed + v)
        for ch in CHANNELS:
            img = getattr(res2, ch)
            up = torch.randn(img.shape, generator=g)
            loss2 = loss2 + (img * up).sum()
        loss2.backward()
        pm2 = res2.projected_means
        out[f"v{v}/projected_means"] = pm.detach().numpy()
        out[f"v{v}/projected_radii"] = res.projected_radii.detach().numpy()
        if sparse:
            rows = np.flatnonzero(
                np.abs(np.concatenate([gr.reshape(n, -1).numpy() for gr in grads], 1)).sum(1) > 0
            )
            out[f"v{v}/rows"] = rows.astype(np.int64)
            for name, gr in zip(names, grads):
                out[f"v{v}/grad_{name}"] = gr.numpy()[rows]
            out[f"v{v}/means2d_grad"] = pm2.grad.numpy()[rows]
            out[f"v{v}/absgrad"] = pm2.absgrad.numpy()[rows]
        else:
            for name, gr in zip(names, grads):
                out[f"v{v}/grad_{name}"] = gr.numpy()
            out[f"v{v}/means2d_grad"] = pm2.grad.numpy()
            out[f"v{v}/absgrad"] = pm2.absgrad.numpy()
    return out


def render_cases():
    from splatforge.studio.batched_renderer import BatchedTorchRenderer
    from splatforge.studio.cameras import Camera
    from splatforge.studio.config import RenderConfig
    from splatforge.studio.renderers import GaussianView, TorchRenderer
    from splatforge_b200 import scenes

    params, cams = scenes.workload("demo48", seed=0)
    cams = cams[:3]
    for mode in ("radegs", "gof", "ambisur"):
        cfg = RenderConfig()
        r = TorchRenderer(cfg, mode=mode, trunc_sigma=2.0)
        out = _run(lambda v, c, s: r.render(v, c, selected=s), params, cams, Camera, GaussianView, 100)
        out["params/" + "means"] = params.means.numpy()
        for name, t in zip(("means", "log_scales", "quats", "opacity_logits", "sh"), params.tensors()):
            out[f"params/{name}"] = t.numpy()
        for v, c in enumerate(cams):
            out[f"cam{v}/K"] = c.K.numpy()
            out[f"cam{v}/w2c"] = c.world_to_camera.numpy()
            out[f"cam{v}/size"] = np.array([c.width, c.height])
        np.savez_compressed(HERE / f"render_{mode}.npz", **out)
        b = BatchedTorchRenderer(cfg, mode=mode, trunc_sigma=2.0)
        out = _run(lambda v, c, s: b.render_training(v, c, selected=s, geometric=True),
                   params, cams[:1], Camera, GaussianView, 200)
        np.savez_compressed(HERE / f"train_{mode}.npz", **out)
    # a tile-aligned crop of a denser surface scene (config-2 distributions)
    params = scenes.surfaces(20_000, seed=3)
    cam = scenes.orbit_cameras(1, 800, 800, 50.0, radius=3.0, seed=3)[0]
    crop = cam.crop(384, 384, 48, 32)
    for mode in ("radegs", "gof"):
        cfg = RenderConfig()
        b = BatchedTorchRenderer(cfg, mode=mode, trunc_sigma=2.0)
        out = _run(lambda v, c, s: b.render(v, c, selected=s, distortions="both"),
                   params, [crop], Camera, GaussianView, 300, sparse=True)
        out["crop/K"] = crop.K.numpy()
        out["crop/w2c"] = crop.world_to_camera.numpy()
        out["crop/size"] = np.array([crop.width, crop.height])
        np.savez_compressed(HERE / f"crop_{mode}.npz", **out)


if __name__ == "__main__":
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPLATFORGE_SRC")
    if not src:
        raise SystemExit("usage: make_golden.py <reference src directory> [fixture ...] (or set SPLATFORGE_SRC)")
    _setup(src)
    which = sys.argv[2:] or ["binning", "ops", "extra", "geometry", "mesh", "training", "render"]
    if "binning" in which:
        binning_cases()
    if "ops" in which:
        op_cases()
    if "geometry" in which:
        geometry_cases()
    if "mesh" in which:
        mesh_cases()
    if "training" in which:
        training_cases()
    if "extra" in which:
        extra_op_cases()
    if "render" in which:
        render_cases()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
