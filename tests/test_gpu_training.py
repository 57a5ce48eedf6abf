"""The training-step kernels (matching.patch_zncc@1, the normal-consistency loss, the
densifier statistics) against the reference's fixtures and the oracle."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import ops as oracle_ops
from splatforge_b200 import ops, training

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def test_patch_zncc_matches_reference(golden):
    """Invalid (short, constant), perfectly correlated, anti-correlated and ordinary
    patches: valid flags exact, correlations within 1e-5, a/b gradients within 1e-4."""
    f = golden("training")
    a = T(f["zncc/a"]).requires_grad_()
    b = T(f["zncc/b"]).requires_grad_()
    corr, valid = ops.patch_zncc(a, b, T(f["zncc/m"]))
    np.testing.assert_array_equal(valid.cpu().numpy(), f["zncc/valid"])
    np.testing.assert_allclose(corr.detach().cpu().numpy(), f["zncc/corr"], atol=1e-5)
    ga, gb = torch.autograd.grad((corr * T(f["zncc/up"])).sum(), (a, b))
    np.testing.assert_allclose(ga.cpu().numpy(), f["zncc/ga"], atol=1e-4)
    np.testing.assert_allclose(gb.cpu().numpy(), f["zncc/gb"], atol=1e-4)


def test_patch_zncc_matches_oracle_on_multiview_sized_batches():
    """[4, 3000, 121] patches (7x7 .. 11x11 windows of a strided pixel grid), leading
    batch dimensions kept, against the oracle's autograd."""
    g = torch.Generator().manual_seed(3)
    a = torch.rand(4, 3000, 121, generator=g)
    b = 0.5 * a + 0.5 * torch.rand(4, 3000, 121, generator=g)
    m = (torch.rand(4, 3000, 121, generator=g) > 0.3).float()
    up = torch.randn(4, 3000, generator=g)
    ac, bc = a.clone().requires_grad_(), b.clone().requires_grad_()
    want, wvalid = oracle_ops.patch_zncc(ac, bc, m)
    wga, wgb = torch.autograd.grad((want * up).sum(), (ac, bc))
    ad, bd = a.to(DEV).requires_grad_(), b.to(DEV).requires_grad_()
    got, gvalid = ops.patch_zncc(ad, bd, m.to(DEV))
    assert got.shape == (4, 3000) and torch.equal(gvalid.cpu(), wvalid)
    np.testing.assert_allclose(got.detach().cpu().numpy(), want.detach().numpy(), atol=2e-6)
    ga, gb = torch.autograd.grad((got * up.to(DEV)).sum(), (ad, bd))
    np.testing.assert_allclose(ga.cpu().numpy(), wga.numpy(), atol=1e-5)
    np.testing.assert_allclose(gb.cpu().numpy(), wgb.numpy(), atol=1e-5)


@pytest.mark.parametrize("tag,numerator", [("num", True), ("unit", False)])
def test_normal_consistency_matches_reference(golden, tag, numerator):
    f = golden("training")
    d = T(f["nc/depth"]).unsqueeze(-1).requires_grad_()
    al = T(f["nc/alpha"]).unsqueeze(-1).requires_grad_()
    v = T(f["nc/nnum" if numerator else "nc/normals"]).requires_grad_()
    out = SimpleNamespace(depth=d, alpha=al, normals=v if not numerator else T(f["nc/normals"]),
                          normal_numerator=v if numerator else None)
    loss = training.normal_consistency(out, SimpleNamespace(K=T(f["nc/K"])), None, T(f["nc/mask"]).unsqueeze(-1))
    np.testing.assert_allclose(loss.item(), f[f"nc/{tag}/loss"], rtol=1e-5)
    gd, gal, gv = torch.autograd.grad(loss * 3.0, (d, al, v), allow_unused=True)
    np.testing.assert_allclose(gd.squeeze(-1).cpu().numpy(), 3.0 * f[f"nc/{tag}/gdepth"], rtol=1e-3, atol=1e-6)
    gal = torch.zeros_like(al) if gal is None else gal
    np.testing.assert_allclose(gal.squeeze(-1).cpu().numpy(), 3.0 * f[f"nc/{tag}/galpha"], rtol=1e-5, atol=1e-9)
    # -g n_depth: near-zero components of the depth normal carry its float rounding
    np.testing.assert_allclose(gv.cpu().numpy(), 3.0 * f[f"nc/{tag}/gvec"], rtol=1e-5, atol=1e-7)


def test_normal_consistency_matches_oracle_at_1080p():
    g = torch.Generator().manual_seed(9)
    H, W = 1080, 1920
    yy, xx = torch.meshgrid(torch.arange(H, dtype=torch.float32), torch.arange(W, dtype=torch.float32), indexing="ij")
    depth = 3.0 + 0.4 * torch.sin(xx / 90.0) * torch.cos(yy / 70.0) + 0.01 * torch.rand(H, W, generator=g)
    alpha = torch.rand(H, W, generator=g)
    nnum = torch.randn(H, W, 3, generator=g) * 0.3
    mask = (torch.rand(H, W, generator=g) > 0.05).float()
    K = torch.tensor([[1662.8, 0.0, 960.0], [0.0, 1662.8, 540.0], [0.0, 0.0, 1.0]])
    dc, vc = depth.clone().requires_grad_(), nnum.clone().requires_grad_()
    want = oracle_ops.normal_consistency(dc, K, alpha, vc, mask, True)
    wd, wv = torch.autograd.grad(want, (dc, vc))
    dd = depth.to(DEV).unsqueeze(-1).requires_grad_()
    vd = nnum.to(DEV).requires_grad_()
    out = SimpleNamespace(depth=dd, alpha=alpha.to(DEV).unsqueeze(-1), normals=None, normal_numerator=vd)
    got = training.normal_consistency(out, SimpleNamespace(K=K), None, mask.to(DEV).unsqueeze(-1))
    np.testing.assert_allclose(got.item(), want.item(), rtol=1e-5)
    gd, gv = torch.autograd.grad(got, (dd, vd))
    rel = (gd.squeeze(-1).cpu() - wd).norm() / wd.norm()
    assert rel < 1e-4, rel
    rel = (gv.cpu() - wv).norm() / wv.norm()
    assert rel < 1e-4, rel


@pytest.mark.parametrize("space", ["pixel", "ndc"])
@pytest.mark.parametrize("absolute", [False, True])
def test_densify_observe_matches_reference(golden, space, absolute):
    f = golden("training")
    n = len(f["dens/radii"])
    dens = SimpleNamespace(config=SimpleNamespace(absolute_gradients=absolute, gradient_space=space),
                           gradient=torch.zeros(n, device=DEV), observations=torch.zeros(n, device=DEV))
    projected = torch.zeros(n, 2, device=DEV)
    projected.grad = T(f["dens/grad"])
    projected.absgrad = T(f["dens/absgrad"])
    out = SimpleNamespace(projected_means=projected, projected_radii=T(f["dens/radii"]),
                          rgb=torch.zeros(24, 40, 3, device=DEV))
    model = SimpleNamespace(count=n)
    for _ in range(2):
        training.observe(dens, out, model)
    key = f"dens/{space}/{'abs' if absolute else 'grad'}"
    np.testing.assert_allclose(dens.gradient.cpu().numpy(), f[f"{key}/gradient"], rtol=1e-6)
    np.testing.assert_array_equal(dens.observations.cpu().numpy(), f[f"{key}/observations"])
    with pytest.raises(ValueError, match="do not match"):
        training.observe(dens, out, SimpleNamespace(count=n + 1))


def test_sh_ambiguity_and_ray_color_variance_match_reference(golden):
    """gaussian.sh_ambiguity@1 and gaussian.ray_color_variance@1/@2 (values and the
    adjoints of seeded linear losses) against the reference."""
    f = golden("ops_extra")
    sh = T(f["amb/sh"]).requires_grad_()
    amb = ops.sh_ambiguity(sh)
    np.testing.assert_allclose(amb.detach().cpu().numpy(), f["amb/out"], rtol=1e-5)
    (g,) = torch.autograd.grad((amb * T(f["amb/up"])).sum(), sh)
    np.testing.assert_allclose(g.cpu().numpy(), f["amb/gsh"], rtol=1e-5, atol=1e-7)
    c = T(f["rcv/c"]).requires_grad_()
    var = ops.ray_color_variance_batch(T(f["rcv/w"]), c, T(f["rcv/r"]))
    np.testing.assert_allclose(var.detach().cpu().numpy(), f["rcv/out"], rtol=1e-5, atol=1e-6)
    (gc,) = torch.autograd.grad((var * T(f["rcv/up"])).sum(), c)
    np.testing.assert_allclose(gc.cpu().numpy(), f["rcv/gc"], rtol=1e-4, atol=1e-5)
    c1 = T(f["rcv/c"][0]).requires_grad_()
    var1 = ops.ray_color_variance(T(f["rcv/w"][0]), c1, T(f["rcv/r"][0]))
    np.testing.assert_allclose(var1.detach().cpu().numpy(), f["rcv/out1"], rtol=1e-5, atol=1e-6)
    (gc1,) = torch.autograd.grad((var1 * T(f["rcv/up"][0])).sum(), c1)
    np.testing.assert_allclose(gc1.cpu().numpy(), f["rcv/gc1"], rtol=1e-4, atol=1e-5)


def test_alpha_composite_v1_and_v2_runners_match_reference(golden):
    """splat.alpha_composite@1 (TorchRenderer's unbatched call) against the reference, and
    @2 against the ops fixture's batched case with both distortions."""
    f = golden("ops_extra")
    ins = [T(f[f"c1/{k}"]).requires_grad_() for k in "acdn"]
    res = ops.alpha_composite(*ins)
    assert len(res) == 8
    for i, r in enumerate(res):
        np.testing.assert_allclose(r.detach().cpu().numpy(), f[f"c1/out{i}"], atol=1e-5)
    loss = sum((r * T(f[f"c1/up{i}"])).sum() for i, r in enumerate(res))
    for k, gr in zip("acdn", torch.autograd.grad(loss, ins)):
        np.testing.assert_allclose(gr.cpu().numpy(), f[f"c1/g{k}"], atol=1e-4)
    g = golden("ops")
    ins = [T(g[f"comp/{k}"]) for k in "acdn"]
    for i, r in enumerate(ops.alpha_composite_batch(*ins)):
        np.testing.assert_allclose(r.cpu().numpy(), g[f"comp/both/out{i}"], atol=1e-5)
