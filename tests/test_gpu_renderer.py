"""The public renderer seam (``render.backend = "b200"``) against the reference's own
fixtures: ``TorchRenderer.render`` and ``BatchedTorchRenderer.render_training`` on the
48-Gaussian demo scene, every mode.  Goes through ``b200_factory`` and
``B200Renderer.render`` / ``render_training`` exactly as the Studio pipelines call them
(src/splatforge/studio/renderers.py:356-439, batched_renderer.py:37-43)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from splatforge_b200 import scenes
from splatforge_b200.renderer import b200_factory
from tests._util import CHANNELS, PARAM_NAMES, camera_from, params_from, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
CONFIG = SimpleNamespace(backend="b200", tile_size=16, sigma_extent=3.0, eps2d=0.3, near=0.01, far=10000.0,
                         background=(1.0, 1.0, 1.0), antialiased=False)


def _view(params):
    """Activation on the CPU (bit-identical inputs to the reference's), then the
    GaussianView fields moved to the device differentiably."""
    p = params.detach_clone().requires_grad_()
    v = scenes.activated(p)
    view = SimpleNamespace(means=v.means.to(DEV), quats=v.quats.to(DEV), scales=v.scales.to(DEV),
                           opacities=v.opacities.to(DEV), sh=v.sh.to(DEV), sh_degree=v.sh_degree)
    return p, view


def _check(fix, out, p, v, profile):
    assert out.distortion_profile == profile
    for ch in CHANNELS:
        got = getattr(out, ch).detach().cpu().numpy()
        want = fix[f"v{v}/{ch}"]
        if ch == "median_depth":
            assert (np.abs(got - want) > 1e-4).mean() <= 0.002, ch
            continue
        # the image bar (1e-4 absolute); L2 is a difference of moments that amplifies
        # the rounding of the reference's LAPACK 2x2 inverse and eigenvalue
        atol = 2e-4 if ch == "distortion_l2" else 1e-4
        rtol = 1e-4 if ch.startswith("distortion") or ch == "depth" else 0.0
        np.testing.assert_allclose(got, want, atol=atol, rtol=rtol, err_msg=f"v{v} {ch}")
    np.testing.assert_allclose(out.projected_means.detach().cpu().numpy(), fix[f"v{v}/projected_means"],
                               atol=1e-4, rtol=1e-5)
    radii = out.projected_radii.detach().cpu().numpy()
    np.testing.assert_allclose(radii, fix[f"v{v}/projected_radii"], rtol=1e-5, atol=1e-5)
    loss = sum((getattr(out, ch) * torch.from_numpy(fix[f"v{v}/up_{ch}"]).to(DEV)).sum() for ch in CHANNELS)
    loss.backward()
    for name, t in zip(PARAM_NAMES, p.tensors()):
        assert rel_err(t.grad.numpy(), fix[f"v{v}/grad_{name}"]) < 1e-3, (v, name)
    xy = out.projected_means
    assert rel_err(xy.grad.cpu().numpy(), fix[f"v{v}/means2d_grad"]) < 1e-3
    assert rel_err(xy.absgrad.cpu().numpy(), fix[f"v{v}/absgrad"]) < 1e-3


@pytest.mark.parametrize("mode", ["radegs", "gof", "ambisur"])
def test_renderer_matches_reference_torch_renderer(golden, mode):
    fix = golden(f"render_{mode}")
    params = params_from(fix)
    renderer = b200_factory(CONFIG, mode=mode, trunc_sigma=2.0, ops=None)
    for v in range(3):
        p, view = _view(params)
        sel = (torch.arange(params.means.shape[0]) % 2 == 0).to(DEV)
        out = renderer.render(view, camera_from(fix, f"cam{v}/"), selected=sel, distortions="both")
        _check(fix, out, p, v, "both")


@pytest.mark.parametrize("mode", ["radegs", "gof", "ambisur"])
def test_render_training_matches_reference_profile(golden, mode):
    fix = golden(f"render_{mode}")
    train = golden(f"train_{mode}")
    params = params_from(fix)
    renderer = b200_factory(CONFIG, mode=mode, trunc_sigma=2.0, ops=None)
    p, view = _view(params)
    sel = (torch.arange(params.means.shape[0]) % 2 == 0).to(DEV)
    out = renderer.render_training(view, camera_from(fix, "cam0/"), selected=sel, geometric=True)
    profile = "none" if mode == "ambisur" else ("l1" if mode == "gof" else "l2")
    _check(train, out, p, 0, profile)
