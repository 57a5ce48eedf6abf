"""The kernels' arithmetic (host build) against the oracle, forward and gradients.

CPU only: ``libsf_b200_hostcheck.so`` runs the projection, per-sample evaluation,
compositing, L1 resolve and every reverse-mode function of the CUDA kernels in
sequential loops.  This pins the hand-written gradients to autograd of the oracle
(which is itself pinned to the reference) before any GPU run.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import render as oracle_render
from splatforge_b200 import scenes
from splatforge_b200.rasterizer import RasterSettings
from tests import hostcheck
from tests._util import CHANNELS, PARAM_NAMES, rel_err

MODES = ("radegs", "gof", "ambisur")


def _oracle(params, cam, mode, distortions, sel, ups):
    p = params.detach_clone().requires_grad_()
    out = oracle_render.render(scenes.activated(p), cam, mode=mode, selected=sel, distortions=distortions)
    loss = sum((out[ch] * ups[ch]).sum() for ch in CHANNELS)
    loss.backward()
    grads = {name: t.grad for name, t in zip(PARAM_NAMES, p.tensors())}
    grads["means2d_grad"] = out["projected_means"].grad
    grads["absgrad"] = out["projected_means"].absgrad
    return out, grads


def _ups(cam, seed):
    g = torch.Generator().manual_seed(seed)
    H, W = cam.height, cam.width
    dims = {"rgb": 3, "normals": 3}
    return {ch: torch.randn(H, W, dims.get(ch, 1), generator=g) for ch in CHANNELS}


def _compare(mode, distortions, params, cam, seed, *, t_stop=0.0, img_tol=2e-5):
    torch.set_num_threads(1)
    n = params.means.shape[0]
    sel = torch.arange(n) % 2 == 0
    ups = _ups(cam, seed)
    settings = RasterSettings(mode=mode, distortions=distortions, transmittance_floor=t_stop)
    want, wgrads = _oracle(params, cam, mode, distortions, sel, ups)
    got, grads, _ = hostcheck.render(params, cam, settings, selected=sel, ups=ups)
    for ch in CHANNELS:
        a, b = got[ch].numpy(), want[ch].detach().numpy()
        if ch == "median_depth":
            bad = np.abs(a - b) > img_tol * (1 + np.abs(b))
            assert bad.mean() <= 0.002, (mode, ch, bad.sum())
            continue
        np.testing.assert_allclose(a, b, atol=img_tol, rtol=1e-4, err_msg=f"{mode}/{distortions} {ch}")
    for name in PARAM_NAMES + ("means2d_grad", "absgrad"):
        e = rel_err(grads[name], wgrads[name])
        assert e < 1e-3, (mode, distortions, name, e)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("distortions", ["none", "l1", "l2", "both"])
def test_hostcheck_demo_scene(mode, distortions):
    params, cams = scenes.workload("demo48", seed=0)
    for v in (0, 3):
        _compare(mode, distortions, params, cams[v], 10 + v)


@pytest.mark.parametrize("mode", ["radegs", "gof"])
def test_hostcheck_surface_crop(mode):
    params = scenes.surfaces(20_000, seed=3)
    cam = scenes.orbit_cameras(1, 800, 800, 50.0, radius=3.0, seed=3)[0].crop(384, 384, 48, 32)
    _compare(mode, "both", params, cam, 7)


def test_hostcheck_early_termination_bound():
    """A transmittance floor of 1e-6 moves no output by more than 1e-5 here."""
    params = scenes.surfaces(20_000, seed=3)
    cam = scenes.orbit_cameras(1, 800, 800, 50.0, radius=3.0, seed=3)[0].crop(384, 384, 48, 32)
    full, _, _ = hostcheck.render(params, cam, RasterSettings(mode="gof", transmittance_floor=0.0))
    cut, _, _ = hostcheck.render(params, cam, RasterSettings(mode="gof", transmittance_floor=1e-6))
    for ch in CHANNELS:
        np.testing.assert_allclose(cut[ch].numpy(), full[ch].numpy(), atol=1e-5, err_msg=ch)


def test_hostcheck_projection_bits_match_oracle():
    """Projected means, radii and camera depth are bit-identical to the oracle's
    exact-sequence projection (they decide tile membership and compositing order)."""
    params = scenes.surfaces(20_000, seed=3)
    cam = scenes.orbit_cameras(1, 800, 800, 50.0, radius=3.0, seed=3)[0]
    _, _, ex = hostcheck.render(params, cam, RasterSettings(mode="gof", distortions="none"))
    view = scenes.activated(params)
    m, _, _, xy, _, filtered = oracle_render.project(view, cam, 0.3, 0.01)
    conic, radii = oracle_render.conic_and_radius(filtered, 3.0)
    assert torch.equal(ex["means2d"], xy)
    assert torch.equal(ex["radii"], radii)
    assert torch.equal(ex["records"][:, 10], m[:, 2])
    assert torch.equal(ex["records"][:, 2], conic[:, 0, 0])
    assert torch.equal(ex["records"][:, 3], conic[:, 0, 1])
    assert torch.equal(ex["records"][:, 4], conic[:, 1, 1])


def test_hostcheck_ambisur_plane_bits_match_oracle():
    """The AmbiSuR camera-facing normal and plane distance (records 11..14) are
    bit-identical to the oracle's: the plane depth plane / (n . ray) amplifies any
    rounding difference at grazing angles, so both evaluate the same exact sequence."""
    params = scenes.surfaces(20_000, seed=5)
    cam = scenes.orbit_cameras(1, 800, 800, 50.0, radius=3.0, seed=5)[0]
    _, _, ex = hostcheck.render(params, cam, RasterSettings(mode="ambisur", distortions="none"))
    view = scenes.activated(params)
    m, _, _, _, _, _ = oracle_render.project(view, cam, 0.3, 0.01)
    normals, plane = oracle_render.ambisur_plane(view, cam, m)
    assert torch.equal(ex["records"][:, 11:14], normals)
    assert torch.equal(ex["records"][:, 14], plane)


def test_warp_cull_never_drops_a_passing_sample():
    """The culling predicate over an 8x4 block of pixel centres is conservative: every
    Gaussian that passes squared <= extent^2 (float32, the kernels' operation order) at
    one of the 32 centres is kept -- for round, elongated and near-degenerate conics."""
    rng = np.random.default_rng(3)
    n = 200_000
    ang = rng.uniform(0, np.pi, n)
    s1 = np.exp(rng.uniform(np.log(0.3), np.log(40.0), n))
    s2 = s1 * np.exp(rng.uniform(np.log(1e-3), 0.0, n))
    c, s = np.cos(ang), np.sin(ang)
    a = c * c / s1**2 + s * s / s2**2
    b = c * s * (1 / s1**2 - 1 / s2**2)
    cc = s * s / s1**2 + c * c / s2**2
    x0, y0 = 100.5, 60.5
    X = x0 + rng.uniform(-60, 68, n)
    Y = y0 + rng.uniform(-60, 64, n)
    g = np.stack([a, b, cc, X, Y], 1).astype(np.float32)
    ext2 = np.float32(9.0)
    keep = hostcheck.box_may_pass(g, (x0, x0 + 7, y0, y0 + 3), 9.0)
    px = (np.float32(x0) + np.arange(8, dtype=np.float32))[None, None, :]
    py = (np.float32(y0) + np.arange(4, dtype=np.float32))[None, :, None]
    qa, qb, qc, gx, gy = (g[:, k][:, None, None] for k in range(5))
    dx, dy = px - gx, py - gy
    sq = dx * (qa * dx + qb * dy) + dy * (qb * dx + qc * dy)
    passes = (sq <= ext2).any((1, 2))
    assert passes.sum() > 1000
    assert not (passes & ~keep).any()
    # and it does cull: most non-passing Gaussians whose bounding box reaches the block
    assert (~keep).sum() > 0.5 * (~passes).sum()
