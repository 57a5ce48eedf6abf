"""Whole frames at the benchmarked sizes: the CUDA path against the oracle run on the
device (tests/_device_oracle.py, the oracle's padded tile batches back-propagated one
batch at a time).

* The million-Gaussian surface scene at 1920x1080 (the first of the bench's poses), in
  all three modes with every output channel and every gradient.
* The view-batched training step's shape: the 3M-Gaussian scene, 8 poses of 1600x1064
  rendered one after another into one accumulated gradient, against the sum of the
  oracle's single-view gradients.  Tile-aligned 128x128 windows of the 8 poses keep
  the oracle's share of the run short; the kernels see the same rays as in the full
  frame.

Bars as everywhere: images 1e-4 absolute (L1/L2 and the AmbiSuR depth also 1e-4
relative; the median may take the neighbouring sample on <= 0.2% of pixels), gradients
1e-3 norm-relative per parameter tensor.
"""

from __future__ import annotations

import time

import pytest
import torch

from splatforge_b200 import scenes
from splatforge_b200.rasterizer import RasterSettings, rasterize
from tests import _device_oracle
from tests._util import CHANNELS, PARAM_NAMES, rel_err
from tests.test_gpu_parity import GRAD_RTOL, _ups, assert_grads, assert_images, run_gpu

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def million_1080p():
    params, cams = scenes.workload("surfaces1m_1080p", seed=0)
    return params, cams[0]


@pytest.mark.parametrize("mode", ["radegs", "gof", "ambisur"])
def test_full_frame_million_gaussians_1080p(million_1080p, mode):
    params, cam = million_1080p
    n = params.means.shape[0]
    sel = torch.arange(n) % 3 == 0
    ups = _ups(cam, 70)
    settings = RasterSettings(mode=mode, distortions="both")
    t0 = time.perf_counter()
    got, ggrads, out = run_gpu(params, cam, settings, sel, ups)
    t1 = time.perf_counter()
    want, wgrads, _ = _device_oracle.render(params, cam, mode, "both", sel, ups, device=DEV)
    t2 = time.perf_counter()
    want = {k: v.cpu() for k, v in want.items()}
    print(f"\n{mode}: {out['n_isect']} intersections; kernels {t1 - t0:.1f} s, device oracle {t2 - t1:.1f} s")
    assert out["n_isect"] > (15_000_000 if mode == "ambisur" else 30_000_000)
    assert_images(got, want, mode, f"1080p/{mode}")
    assert_grads(ggrads, wgrads, f"1080p/{mode}")


def test_view_batched_step_accumulates_eight_views():
    params, cams = scenes.workload("surfaces3m_views64", seed=0)
    poses = cams[:8]
    windows = [c.crop(736, 464, 128, 128) for c in poses]
    settings = RasterSettings(mode="gof", distortions="l1")
    ups = [_ups(c, 900 + k) for k, c in enumerate(windows)]

    # the training step as bench.py runs it: device parameters, one render + backward
    # per pose, gradients accumulating on the parameters across the poses
    p = params.to(DEV).requires_grad_()
    for cam, up in zip(windows, ups):
        v = scenes.activated(p)
        out = rasterize(v.means, v.quats, v.scales, v.opacities, v.sh, 3, cam, settings)
        sum((out[ch] * up[ch].to(DEV)).sum() for ch in CHANNELS).backward()
        assert int(out["plan"].error_word.item()) == 0
    got = {name: t.grad.cpu() for name, t in zip(PARAM_NAMES, p.tensors())}

    want = {name: torch.zeros_like(t) for name, t in zip(PARAM_NAMES, params.tensors())}
    for cam, up in zip(windows, ups):
        _, g, _ = _device_oracle.render(params, cam, "gof", "l1", None, up, device=DEV, activation_device=DEV)
        for name in PARAM_NAMES:
            want[name] += g[name].cpu()
    for name in PARAM_NAMES:
        e = rel_err(got[name], want[name])
        assert e < GRAD_RTOL, (name, e)
