"""The batch-by-batch oracle helper (tests/_device_oracle.py) equals the oracle's
whole-frame graph: same images, same gradients, on the CPU."""

from __future__ import annotations

import torch

from oracle import render as oracle_render
from splatforge_b200 import scenes
from tests import _device_oracle
from tests._util import CHANNELS, PARAM_NAMES, rel_err


def _ups(cam, seed):
    g = torch.Generator().manual_seed(seed)
    return {ch: torch.randn(cam.height, cam.width, 3 if ch in ("rgb", "normals") else 1, generator=g)
            for ch in CHANNELS}


def _whole(params, cam, mode, distortions, sel, ups):
    p = params.detach_clone().requires_grad_()
    out = oracle_render.render(scenes.activated(p), cam, mode=mode, selected=sel, distortions=distortions)
    sum((out[ch] * ups[ch]).sum() for ch in CHANNELS).backward()
    grads = {name: t.grad for name, t in zip(PARAM_NAMES, p.tensors())}
    grads["means2d_grad"] = out["projected_means"].grad
    grads["absgrad"] = out["projected_means"].absgrad
    return {ch: out[ch].detach() for ch in CHANNELS}, grads


def test_batched_helper_equals_the_whole_frame_graph():
    torch.set_num_threads(4)
    params, cams = scenes.workload("demo48", seed=0)
    sel = torch.arange(48) % 2 == 0
    for mode, v in (("gof", 0), ("radegs", 3), ("ambisur", 5)):
        cam = cams[v]
        ups = _ups(cam, 50 + v)
        want, wg = _whole(params, cam, mode, "both", sel, ups)
        got, gg, _ = _device_oracle.render(params, cam, mode, "both", sel, ups, device="cpu")
        for ch in CHANNELS:
            assert torch.allclose(got[ch], want[ch], atol=1e-6, rtol=1e-6), (mode, ch)
        for name in PARAM_NAMES + ("means2d_grad", "absgrad"):
            assert rel_err(gg[name], wg[name]) < 1e-5, (mode, name)


def test_batched_helper_on_a_surface_crop():
    torch.set_num_threads(8)
    params, cams = scenes.workload("surfaces100k_800", seed=0)
    cam = cams[0].crop(384, 384, 32, 32)
    ups = _ups(cam, 5)
    want, wg = _whole(params, cam, "gof", "both", None, ups)
    got, gg, _ = _device_oracle.render(params, cam, "gof", "both", None, ups, device="cpu")
    for ch in CHANNELS:
        assert torch.allclose(got[ch], want[ch], atol=1e-6, rtol=1e-6), ch
    for name in PARAM_NAMES + ("means2d_grad", "absgrad"):
        assert rel_err(gg[name], wg[name]) < 1e-5, name
