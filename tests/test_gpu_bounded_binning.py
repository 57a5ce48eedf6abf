"""Binning without the count read-back (``sf_b200_bin_emit_bounded``).

The first render of a (Gaussian count, image size) bins with the exact intersection
count; later ones size the lists by the learned capacity and read the count back
together with the forward's other flags.  Rendering the same view twice must give the
same lists and the same images bit for bit, and a capacity that is too small must be
caught and re-binned with the result unchanged.
"""

from __future__ import annotations

import pytest
import torch

from splatforge_b200 import rasterizer, scenes
from splatforge_b200.rasterizer import RasterSettings
from tests._util import CHANNELS, rel_err
from tests.test_gpu_parity import _ups, run_gpu

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _render(params, cam, distortions):
    ups = _ups(cam, 5)
    return run_gpu(params, cam, RasterSettings(mode="gof", distortions=distortions), None, ups)


def _bin_key(params, cam):
    return (params.means.shape[0], cam.width, cam.height)


@pytest.mark.parametrize("distortions", ["both", "none"])
def test_bounded_binning_equals_exact_binning(distortions):
    params, cams = scenes.workload("surfaces100k_800", seed=0)
    cam = cams[0].crop(256, 256, 160, 128)
    rasterizer._ISECT_SEEN.pop(_bin_key(params, cam), None)
    imgs0, grads0, out0 = _render(params, cam, distortions)  # exact: learns the capacity
    assert _bin_key(params, cam) in rasterizer._ISECT_SEEN
    ids0 = out0["plan"].ids[: out0["n_isect"]].clone()
    imgs1, grads1, out1 = _render(params, cam, distortions)  # bounded
    assert out1["n_isect"] == out0["n_isect"] > 0
    assert out1["plan"].ids.numel() > out1["n_isect"]  # sized by the capacity
    assert torch.equal(out1["plan"].ids[: out1["n_isect"]], ids0)
    assert torch.equal(out1["plan"].ranges, out0["plan"].ranges)
    for ch in CHANNELS:
        assert torch.equal(imgs1[ch], imgs0[ch]), ch
    for name in grads0:
        # the same sums in another order (float atomics; the quaternion gradient sums
        # terms that cancel): norm-relative, 10x inside the oracle bar
        assert rel_err(grads1[name], grads0[name]) < 1e-4, name


def test_capacity_overflow_is_rebinned():
    params, cams = scenes.workload("surfaces100k_800", seed=0)
    cam = cams[0].crop(128, 384, 192, 96)
    key = _bin_key(params, cam)
    rasterizer._ISECT_SEEN.pop(key, None)
    imgs0, grads0, out0 = _render(params, cam, "both")
    rasterizer._ISECT_SEEN[key] = 1024  # far below the count
    reruns = rasterizer.COUNTERS["bin_reruns"]
    imgs1, grads1, out1 = _render(params, cam, "both")
    assert rasterizer.COUNTERS["bin_reruns"] == reruns + 1
    assert out1["stats"].get("bin_rerun")
    assert out1["n_isect"] == out0["n_isect"] > 1024
    assert rasterizer._ISECT_SEEN[key] >= out0["n_isect"]  # the capacity grew
    for ch in CHANNELS:
        assert torch.equal(imgs1[ch], imgs0[ch]), ch
    for name in grads0:
        # the same sums in another order (float atomics; the quaternion gradient sums
        # terms that cancel): norm-relative, 10x inside the oracle bar
        assert rel_err(grads1[name], grads0[name]) < 1e-4, name
