"""Operator runners (gaussian.covariance@1, gaussian.sh_color@1,
splat.alpha_composite@3, gaussian.opacity_field@1) on the GPU against the reference's
golden fixtures and the CPU oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oracle_ops
from splatforge_b200 import ops
from tests._util import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(a, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t.requires_grad_() if grad else t


def test_covariance_matches_reference_fixture_and_gradients(golden):
    f = golden("ops")
    q, s = T(f["cov/quats"], True), T(f["cov/scales"], True)
    cov = ops.covariance(q, s)
    np.testing.assert_allclose(cov.detach().cpu().numpy(), f["cov/out"], atol=1e-6)
    g = torch.randn(cov.shape, generator=torch.Generator().manual_seed(3)).to(DEV)
    gq, gs = torch.autograd.grad((cov * g).sum(), (q, s))
    qc, sc = torch.from_numpy(f["cov/quats"]).requires_grad_(), torch.from_numpy(f["cov/scales"]).requires_grad_()
    wq, ws = torch.autograd.grad((oracle_ops.covariance(qc, sc) * g.cpu()).sum(), (qc, sc))
    assert rel_err(gq.cpu(), wq) < 1e-4 and rel_err(gs.cpu(), ws) < 1e-4


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_sh_color_matches_reference_fixture(golden, degree):
    f = golden("ops")
    sh, d = T(f["sh/coeffs"], True), T(f["sh/dirs"], True)
    col = ops.sh_color(sh, d, degree=degree)
    np.testing.assert_allclose(col.detach().cpu().numpy(), f[f"sh/deg{degree}/out"], atol=1e-6)
    gs, gd = torch.autograd.grad((col * T(f[f"sh/deg{degree}/up"])).sum(), (sh, d))
    np.testing.assert_allclose(gs.cpu().numpy(), f[f"sh/deg{degree}/gcoeffs"], atol=1e-6)
    np.testing.assert_allclose(gd.cpu().numpy(), f[f"sh/deg{degree}/gdirs"], atol=2e-5)


@pytest.mark.parametrize("profile", ["none", "l1", "l2", "both"])
def test_alpha_composite_matches_reference_fixture(golden, profile):
    """Includes alphas clamped at 0.999 and at 0 (no adjoint through the clamp)."""
    f = golden("ops")
    ins = [T(f[f"comp/{k}"], True) for k in "acdn"]
    res = ops.alpha_composite_selected(*ins, distortions=profile)
    for i, r in enumerate(res):
        # L2 (out5) is a difference of moments ~4 accumulated in another order
        atol = 2e-5 if i == 5 else 2e-6
        np.testing.assert_allclose(r.detach().cpu().numpy(), f[f"comp/{profile}/out{i}"], atol=atol, rtol=1e-5,
                                   err_msg=f"out{i}")
    loss = sum((r * T(f[f"comp/up{i}"])).sum() for i, r in enumerate(res))
    grads = torch.autograd.grad(loss, ins)
    for name, g in zip("acdn", grads):
        np.testing.assert_allclose(g.cpu().numpy(), f[f"comp/{profile}/g{name}"], atol=5e-5, err_msg=name)


@pytest.mark.parametrize("profile", ["l1", "both"])
def test_alpha_composite_large_against_oracle(profile):
    g = torch.Generator().manual_seed(11)
    B, N, P = 4, 300, 256
    a = (torch.rand(B, N, P, generator=g) * 0.3)
    c = torch.rand(B, N, 3, generator=g)
    d = torch.rand(B, N, P, generator=g) * 3 + 1
    n = torch.randn(B, N, P, 3, generator=g)
    ups = None
    outs = {}
    for side in ("gpu", "cpu"):
        ins = [t.clone().to(DEV if side == "gpu" else "cpu").requires_grad_() for t in (a, c, d, n)]
        fn = ops.alpha_composite_selected if side == "gpu" else oracle_ops.alpha_composite_batch
        res = fn(*ins, distortions=profile)
        if ups is None:
            ups = [torch.randn(r.shape, generator=g) for r in res]
        loss = sum((r * u.to(r.device)).sum() for r, u in zip(res, ups))
        outs[side] = ([r.detach().cpu() for r in res], [x.cpu() for x in torch.autograd.grad(loss, ins)])
    for i, (x, y) in enumerate(zip(outs["gpu"][0], outs["cpu"][0])):
        np.testing.assert_allclose(x.numpy(), y.numpy(), atol=1e-4, rtol=1e-4, err_msg=f"out{i}")
    for name, x, y in zip("acdn", outs["gpu"][1], outs["cpu"][1]):
        assert rel_err(x, y) < 1e-3, name


def test_composite_rejects_cpu_and_bad_profile():
    x = torch.rand(1, 2, 3)
    with pytest.raises(ValueError):
        ops.alpha_composite_selected(x, torch.rand(1, 2, 3), x, torch.rand(1, 2, 3, 3), distortions="both")
    with pytest.raises(ValueError):
        y = x.to(DEV)
        ops.alpha_composite_selected(y, torch.rand(1, 2, 3, device=DEV), y, torch.rand(1, 2, 3, 3, device=DEV),
                                     distortions="l3")


def test_opacity_field_matches_reference_fixture(golden):
    f = golden("ops")
    out = ops.opacity_field(*(T(f[f"field/{k}"]) for k in ("p", "m", "Q", "o", "origins")))
    np.testing.assert_allclose(out.cpu().numpy(), f["field/out"], atol=1e-6)


def test_opacity_field_larger_against_oracle():
    g = torch.Generator().manual_seed(5)
    P, N, C = 3000, 2000, 5
    pts = torch.randn(P, 3, generator=g) * 0.7
    m = torch.randn(N, 3, generator=g) * 0.6
    L = torch.randn(N, 3, 3, generator=g) * 0.05
    cov = L @ L.transpose(-1, -2) + 1e-3 * torch.eye(3)
    Q = torch.linalg.inv(cov)
    op = torch.rand(N, generator=g)
    origins = torch.randn(C, 3, generator=g) * 3
    want = oracle_ops.opacity_field(pts, m, Q, op, origins)
    got = ops.opacity_field(*(t.to(DEV) for t in (pts, m, Q, op, origins)))
    np.testing.assert_allclose(got.cpu().numpy(), want.numpy(), atol=2e-5)


def _field_case(n, n_uniform, n_views, seed=0):
    from splatforge_b200 import scenes

    params = scenes.surfaces(n, seed)
    v = scenes.activated(params)
    Q = scenes.inverse_covariances(params)
    pts = scenes.field_queries(params, n_uniform, seed=seed)
    cams = scenes.orbit_cameras(n_views, 64, 64, 60.0, radius=3.0, seed=seed)
    origins = torch.stack([c.origin for c in cams])
    return pts, v.means.contiguous(), Q.contiguous(), v.opacities.contiguous(), origins


def _brute(*args):
    return ops.opacity_field(*args)


def test_opacity_field_culled_matches_brute_force():
    """The culled field (per-view cube-map candidate lists, contributions <= 1e-7
    dropped) against the brute-force kernel on an exporter-shaped query set:
    9 points per Gaussian of a 20k surface scene plus 20k uniform points, 6 views."""
    args = [t.to(DEV) for t in _field_case(20_000, 20_000, 6)]
    full = _brute(*args)
    cull = ops.opacity_field_culled(*args)
    assert torch.isfinite(cull).all()
    assert (full - cull).abs().max().item() < 1e-5
    assert full.max().item() > 0.5  # the grid does reach dense regions


def test_opacity_field_culled_edge_cases_against_oracle():
    """An origin inside a Gaussian's bounding ball (its global list), a query at an
    origin (no direction: zero field for that view), a Gaussian below the cutoff, and
    a wide face_cells range, against the oracle."""
    pts, m, Q, o, org = _field_case(300, 400, 3, seed=4)
    org = torch.cat((org, m[7:8] + 1e-3), 0)                # origin inside Gaussian 7
    pts = torch.cat((pts, org[1:2], m[7:8] + 2e-3), 0)        # a query at origin 1
    o = o.clone()
    o[11] = 5e-8                                               # below the cutoff
    want = oracle_ops.opacity_field(pts, m, Q, o, org)
    for cells in (1, 16, 128):
        got = ops.opacity_field_culled(*(t.to(DEV) for t in (pts, m, Q, o, org)), face_cells=cells)
        np.testing.assert_allclose(got.cpu().numpy(), want.numpy(), atol=2e-5, err_msg=f"face_cells={cells}")
    assert want[-2].item() == 0.0


def test_opacity_field_plan_equals_the_culled_field():
    """The plan (all views' lists built once, all views' queries in one pass) gives the
    culled field's values bit for bit, on the 20k scene and on the edge cases (origin
    inside a Gaussian's ball, a query at an origin, a Gaussian below the cutoff), and
    stays valid across calls with different query sets."""
    args = [t.to(DEV) for t in _field_case(20_000, 20_000, 6)]
    plan = ops.OpacityFieldPlan(*args[1:])
    assert torch.equal(plan(args[0]), ops.opacity_field_culled(*args))
    part = args[0][::7].contiguous()
    assert torch.equal(plan(part), ops.opacity_field_culled(part, *args[1:]))
    pts, m, Q, o, org = _field_case(300, 400, 3, seed=4)
    org = torch.cat((org, m[7:8] + 1e-3), 0)
    pts = torch.cat((pts, org[1:2], m[7:8] + 2e-3), 0)
    o = o.clone()
    o[11] = 5e-8
    d = [t.to(DEV) for t in (pts, m, Q, o, org)]
    for cells in (1, 16, 128):
        got = ops.OpacityFieldPlan(*d[1:], face_cells=cells)(d[0])
        assert torch.equal(got, ops.opacity_field_culled(*d, face_cells=cells)), cells
    assert got[-2].item() == 0.0
    empty = ops.OpacityFieldPlan(d[1][:0], d[2][:0], d[3][:0], d[4])
    assert torch.equal(empty(d[0]), ops.opacity_field(d[0], d[1][:0], d[2][:0], d[3][:0], d[4]))


def test_opacity_field_culled_reference_fixture(golden):
    f = golden("ops")
    out = ops.opacity_field_culled(*(T(f[f"field/{k}"]) for k in ("p", "m", "Q", "o", "origins")))
    np.testing.assert_allclose(out.cpu().numpy(), f["field/out"], atol=1e-5)


def test_geometry_ops_match_reference_fixture(golden):
    """camera.pixel_rays@1, gaussian.ray_peak@1 and geometry.depth_normals@1 (with the
    depth adjoint) against the reference's outputs."""
    f = golden("geometry")
    np.testing.assert_allclose(ops.pixel_rays(T(f["rays/K"]), width=64, height=48).cpu().numpy(), f["rays/out"],
                               atol=1e-6)
    t, r, n = ops.ray_peak(*(T(f[f"peak/{k}"]) for k in ("means", "Q", "o", "d")))
    np.testing.assert_allclose(t.cpu().numpy(), f["peak/t"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r.cpu().numpy(), f["peak/r"], atol=1e-6)
    np.testing.assert_allclose(n.cpu().numpy(), f["peak/n"], atol=1e-6)
    depth = T(f["dn/depth"], True)
    normals, valid = ops.depth_normals(depth, T(f["dn/K"]))
    np.testing.assert_array_equal(valid.cpu().numpy(), f["dn/valid"])
    np.testing.assert_allclose(normals.detach().cpu().numpy(), f["dn/normals"], atol=1e-6)
    (gd,) = torch.autograd.grad((normals * T(f["dn/up"])).sum(), depth)
    np.testing.assert_allclose(gd.cpu().numpy(), f["dn/gdepth"], rtol=1e-4, atol=1e-5)


def test_depth_normals_full_frame_against_oracle():
    """A 1080p depth map with holes: normals, validity and the depth adjoint."""
    g = torch.Generator().manual_seed(3)
    H, W = 1080, 1920
    yy, xx = torch.meshgrid(torch.arange(H, dtype=torch.float32), torch.arange(W, dtype=torch.float32), indexing="ij")
    depth = 3.0 + 0.5 * torch.sin(xx / 90.0) * torch.cos(yy / 70.0) + 0.01 * torch.rand(H, W, generator=g)
    depth[torch.rand(H, W, generator=g) < 0.01] = 0.0
    K = torch.tensor([[1662.8, 0.0, 960.0], [0.0, 1662.8, 540.0], [0.0, 0.0, 1.0]])
    up = torch.randn(H, W, 3, generator=g)
    dc = depth.clone().requires_grad_()
    wn, wv = oracle_ops.depth_normals(dc, K)
    (wg,) = torch.autograd.grad((wn * up).sum(), dc)
    dg = depth.to(DEV).requires_grad_()
    gn, gv = ops.depth_normals(dg, K.to(DEV))
    (gg,) = torch.autograd.grad((gn * up.to(DEV)).sum(), dg)
    assert (gv.cpu() == wv).float().mean().item() > 0.9999
    both = (gv.cpu() & wv).unsqueeze(-1)
    np.testing.assert_allclose((gn.detach().cpu() * both).numpy(), (wn.detach() * both).numpy(), atol=1e-4)
    assert rel_err(gg.cpu(), wg) < 1e-3
