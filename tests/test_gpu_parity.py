"""CUDA path (libsf_b200.so through the C ABI) against the CPU oracle.

Targets: tile lists and sorted keys bit-exact; forward images within 1e-4 absolute
(float32); gradients within 1e-3 relative (norm-relative per parameter tensor).
Discontinuities the reference itself has are handled explicitly: the median depth
may pick the neighbouring sample where the cumulative weight sits within float
rounding of 0.5 (a bounded fraction of pixels), and the AmbiSuR plane depth is a
ratio with a small denominator, compared with a relative term.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import binning as oracle_binning
from oracle import render as oracle_render
from splatforge_b200 import scenes
from splatforge_b200.rasterizer import RasterSettings, rasterize
from tests._util import CHANNELS, PARAM_NAMES, rel_err

pytestmark = pytest.mark.gpu

DEV = "cuda"
IMG_ATOL = 1e-4
GRAD_RTOL = 1e-3


def _ups(cam, seed):
    g = torch.Generator().manual_seed(seed)
    dims = {"rgb": 3, "normals": 3}
    return {ch: torch.randn(cam.height, cam.width, dims.get(ch, 1), generator=g) for ch in CHANNELS}


def run_gpu(params, cam, settings, sel, ups):
    """The activation (exp / sigmoid) runs on the CPU and the activated tensors are
    copied to the device differentiably, so both paths see bit-identical inputs
    (torch's CUDA and CPU exp can differ in the last bit)."""
    p = params.detach_clone().requires_grad_()
    v = scenes.activated(p)
    view = [t.to(DEV) for t in (v.means, v.quats, v.scales, v.opacities, v.sh)]
    out = rasterize(*view, params.sh_degree, cam, settings, selected=None if sel is None else sel.to(DEV))
    loss = sum((out[ch] * ups[ch].to(DEV)).sum() for ch in CHANNELS)
    loss.backward()
    grads = {name: t.grad.cpu() for name, t in zip(PARAM_NAMES, p.tensors())}
    grads["means2d_grad"] = out["projected_means"].grad.cpu()
    grads["absgrad"] = out["projected_means"].absgrad.cpu()
    imgs = {ch: out[ch].detach().cpu() for ch in CHANNELS}
    # the backward's recomputed contributing samples matched the forward's count
    assert int(out["plan"].error_word.item()) == 0
    return imgs, grads, out


def run_oracle(params, cam, mode, distortions, sel, ups, settings=None):
    p = params.detach_clone().requires_grad_()
    out = oracle_render.render(scenes.activated(p), cam, mode=mode, selected=sel, distortions=distortions,
                               settings=settings)
    loss = sum((out[ch] * ups[ch]).sum() for ch in CHANNELS)
    loss.backward()
    grads = {name: t.grad for name, t in zip(PARAM_NAMES, p.tensors())}
    grads["means2d_grad"] = out["projected_means"].grad
    grads["absgrad"] = out["projected_means"].absgrad
    return {ch: out[ch].detach() for ch in CHANNELS}, grads, out


def assert_images(got, want, mode, tag):
    for ch in CHANNELS:
        a, b = got[ch].numpy(), want[ch].numpy()
        assert np.isfinite(a).all(), (tag, ch)
        if ch == "median_depth":
            bad = np.abs(a - b) > IMG_ATOL
            assert bad.mean() <= 0.002, (tag, ch, int(bad.sum()))
            continue
        # AmbiSuR expected depth divides by n.ray; L2 is a difference of moments:
        # both scale the same float32 rounding by their magnitude
        rtol = 1e-4 if (ch == "depth" and mode == "ambisur") or ch.startswith("distortion") else 0.0
        np.testing.assert_allclose(a, b, atol=IMG_ATOL, rtol=rtol, err_msg=f"{tag} {ch}")


def assert_grads(got, want, tag):
    for name in PARAM_NAMES + ("means2d_grad", "absgrad"):
        e = rel_err(got[name], want[name])
        assert e < GRAD_RTOL, (tag, name, e)


@pytest.mark.parametrize("mode", ["radegs", "gof", "ambisur"])
@pytest.mark.parametrize("distortions", ["none", "l1", "l2", "both"])
def test_demo_scene_all_views(mode, distortions):
    torch.set_num_threads(4)
    params, cams = scenes.workload("demo48", seed=0)
    sel = torch.arange(48) % 2 == 0
    settings = RasterSettings(mode=mode, distortions=distortions)
    for v, cam in enumerate(cams):
        ups = _ups(cam, 100 + v)
        got, ggrads, _ = run_gpu(params, cam, settings, sel, ups)
        want, wgrads, _ = run_oracle(params, cam, mode, distortions, sel, ups)
        assert_images(got, want, mode, f"{mode}/{distortions}/v{v}")
        assert_grads(ggrads, wgrads, f"{mode}/{distortions}/v{v}")


CROPS = {
    "surfaces100k_800": [(384, 384, 64, 64), (160, 512, 48, 32)],
    "surfaces1m_1080p": [(928, 512, 64, 64), (400, 304, 48, 48)],
}


@pytest.mark.parametrize("workload", list(CROPS))
@pytest.mark.parametrize("mode", ["radegs", "gof", "ambisur"])
def test_surface_scene_crops(workload, mode):
    """Tile-aligned crops (principal point shifted by multiples of 16): same rays as
    the full frame for the covered pixels."""
    torch.set_num_threads(8)
    params, cams = scenes.workload(workload, seed=0)
    n = params.means.shape[0]
    sel = torch.arange(n) % 3 == 0
    settings = RasterSettings(mode=mode, distortions="both")
    for k, (left, top, w, h) in enumerate(CROPS[workload]):
        cam = cams[0].crop(left, top, w, h)
        ups = _ups(cam, 7 + k)
        got, ggrads, _ = run_gpu(params, cam, settings, sel, ups)
        want, wgrads, _ = run_oracle(params, cam, mode, "both", sel, ups)
        assert_images(got, want, mode, f"{workload}/{mode}/crop{k}")
        assert_grads(ggrads, wgrads, f"{workload}/{mode}/crop{k}")


def test_forward_is_bitwise_repeatable_and_projection_matches():
    params, cams = scenes.workload("surfaces100k_800", seed=0)
    cam = cams[0]
    settings = RasterSettings(mode="gof", distortions="both")
    v = scenes.activated(params)
    view = scenes.View(*(t.to(DEV) for t in (v.means, v.quats, v.scales, v.opacities, v.sh)), 3)
    with torch.no_grad():
        a = rasterize(view.means, view.quats, view.scales, view.opacities, view.sh, 3, cam, settings)
        b = rasterize(view.means, view.quats, view.scales, view.opacities, view.sh, 3, cam, settings)
    for ch in CHANNELS:
        assert torch.equal(a[ch], b[ch]), ch
    # projected means / radii are the oracle's exact-sequence values bit for bit
    m, _, _, xy, _, filt = oracle_render.project(scenes.activated(params), cam, 0.3, 0.01)
    _, radii = oracle_render.conic_and_radius(filt, 3.0)
    assert torch.equal(a["projected_means"].cpu(), xy)
    assert torch.equal(a["projected_radii"].cpu(), radii)


# ---------------------------------------------------------------- binning through the C ABI
def _bin_device(bounds, width, height, near, far):
    from splatforge_b200 import _lib
    from splatforge_b200.rasterizer import _ptr, _stream

    b = torch.from_numpy(np.ascontiguousarray(bounds, dtype=np.float32)).to(DEV)
    n = b.shape[0]
    rect = torch.empty((n, 4), device=DEV, dtype=torch.int32)
    count = torch.empty((n,), device=DEV, dtype=torch.int32)
    dkey = torch.empty((n,), device=DEV, dtype=torch.int32)
    nonfinite = torch.zeros((1,), device=DEV, dtype=torch.int32)
    st = _stream(torch.device(DEV))
    _lib.call("sf_b200_bin_rects", ctypes.c_void_p(b.data_ptr()), n, width, height, 16, near, far,
              _ptr(rect), _ptr(count), _ptr(dkey), _ptr(nonfinite), st)
    tx, ty = (width + 15) // 16, (height + 15) // 16
    T = tx * ty
    size = ctypes.c_size_t()
    _lib.call("sf_b200_bin_workspace_bytes", n, 0, T, ctypes.byref(size))
    ws = torch.empty((max(size.value, 1),), device=DEV, dtype=torch.uint8)
    order = torch.empty((n,), device=DEV, dtype=torch.int32)
    offsets = torch.empty((n + 1,), device=DEV, dtype=torch.int64)
    _lib.call("sf_b200_bin_order", _ptr(count), _ptr(dkey), n, _ptr(order), _ptr(offsets), _ptr(ws), size.value, st)
    m = int(offsets[n].item())
    _lib.call("sf_b200_bin_workspace_bytes", n, m, T, ctypes.byref(size))
    ws = torch.empty((max(size.value, 1),), device=DEV, dtype=torch.uint8)
    ids = torch.empty((max(m, 1),), device=DEV, dtype=torch.int32)
    ranges = torch.empty((T, 2), device=DEV, dtype=torch.int32)
    _lib.call("sf_b200_bin_emit", _ptr(order), _ptr(offsets), _ptr(rect), n, m, tx, T, _ptr(ids), _ptr(ranges),
              _ptr(ws), size.value, st)
    keys = torch.empty((max(m, 1),), device=DEV, dtype=torch.int64)
    _lib.call("sf_b200_bin_keys", _ptr(ids), _ptr(ranges), _ptr(dkey), T, m, _ptr(keys), st)
    r = ranges.cpu().numpy().astype(np.int64)
    offs = np.zeros(T + 1, dtype=np.int64)
    counts = r[:, 1] - r[:, 0]
    offs[1:] = np.cumsum(counts)
    # tiles with members start where the previous ended
    assert np.all(r[counts > 0, 0] == offs[:-1][counts > 0])
    return offs, ids.cpu().numpy()[:m].astype(np.int64), keys.cpu().numpy()[:m].view(np.uint64), int(nonfinite.item())


@pytest.mark.parametrize("case", ["fixture703", "random0", "random1"])
def test_binning_bit_exact_against_reference_fixtures(golden, case):
    fix = golden("binning")
    w, h, ts, near, far = fix[f"{case}/meta"]
    offs, ids, keys, bad = _bin_device(fix[f"{case}/bounds"], int(w), int(h), float(near), float(far))
    assert bad == 0
    np.testing.assert_array_equal(offs, fix[f"{case}/offsets"])
    np.testing.assert_array_equal(ids, fix[f"{case}/ids"])
    _, _, want_keys = oracle_binning.tile_lists(fix[f"{case}/bounds"], width=int(w), height=int(h), tile_size=16,
                                                near=near, far=far)
    np.testing.assert_array_equal(keys, want_keys)


def test_binning_bit_exact_full_frame_million():
    """1M-Gaussian 1080p bounds: every tile list and 64-bit key equal to the oracle."""
    params, cams = scenes.workload("surfaces1m_1080p", seed=0)
    cam = cams[0]
    m, _, _, xy, _, filt = oracle_render.project(scenes.activated(params), cam, 0.3, 0.01)
    _, radii = oracle_render.conic_and_radius(filt, 3.0)
    bounds = torch.cat((xy, radii[:, None], m[:, 2:3]), 1).numpy()
    offs, ids, keys, bad = _bin_device(bounds, cam.width, cam.height, 0.01, 1e4)
    want_offs, want_ids, want_keys = oracle_binning.tile_lists(bounds, width=cam.width, height=cam.height,
                                                               tile_size=16, near=0.01, far=1e4)
    assert bad == 0
    np.testing.assert_array_equal(offs, want_offs)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(keys, want_keys)


def test_nonfinite_bounds_raise():
    bounds = np.array([[10, 10, 3, 2], [np.nan, 3, 1, 2], [5, 5, np.inf, 1]], np.float32)
    _, _, _, bad = _bin_device(bounds, 32, 32, 0.01, 1e4)
    assert bad == 2


def test_empty_scene_is_background():
    cam = scenes.orbit_cameras(1, 40, 24, 60.0)[0]
    z = torch.zeros((0, 3), device=DEV)
    out = rasterize(z, torch.zeros((0, 4), device=DEV), z, torch.zeros((0,), device=DEV),
                    torch.zeros((0, 16, 3), device=DEV), 3, cam, RasterSettings(mode="gof", background=(0.2, 0.3, 0.4)))
    assert torch.allclose(out["rgb"], torch.tensor([0.2, 0.3, 0.4], device=DEV).expand(24, 40, 3))
    assert float(out["alpha"].abs().max()) == 0.0
    assert out["n_isect"] == 0


def test_l1_capacity_overflow_reruns_with_exact_storage():
    params, cams = scenes.workload("surfaces100k_800", seed=0)
    cam = cams[0].crop(384, 384, 32, 32)
    sel = torch.arange(params.means.shape[0]) % 2 == 0
    ups = _ups(cam, 3)
    small = RasterSettings(mode="gof", distortions="l1", l1_capacity=32)
    big = RasterSettings(mode="gof", distortions="l1", l1_capacity=1024)
    a, ga, out = run_gpu(params, cam, small, sel, ups)
    b, gb, outb = run_gpu(params, cam, big, sel, ups)
    assert out["stats"]["l1_max_samples"] > 32 and out["stats"].get("l1_rerun")
    assert not outb["stats"].get("l1_rerun")
    for ch in CHANNELS:
        np.testing.assert_allclose(a[ch].numpy(), b[ch].numpy(), atol=1e-6)
    for name in PARAM_NAMES:
        assert rel_err(ga[name], gb[name]) < 1e-5


def test_cpu_inputs_are_rejected_without_fallback():
    params, cams = scenes.workload("demo48", seed=0)
    view = scenes.activated(params)
    with pytest.raises(ValueError):
        rasterize(view.means, view.quats, view.scales, view.opacities, view.sh, 3, cams[0], RasterSettings())


@pytest.mark.parametrize("n,opacity,lo,hi", [
    (420, 0.004, 257, 512),     # 16 samples per lane, one warp per pixel
    (700, 0.004, 513, 1024),    # one CTA per pixel, 4 samples per thread in registers
    (1500, 0.004, 1025, 2048),  # 8 per thread
    (3000, 0.002, 2049, 4096),  # 16 per thread
    (5000, 0.002, 4097, 8192),  # the shared-memory network
])
def test_l1_long_sample_runs_match_the_oracle(n, opacity, lo, hi):
    """n faint, wide Gaussians over a 32x24 image: every pixel composites up to n
    samples (transmittance stays above the floor), which takes each sort of the L1
    resolve in turn as the runs grow."""
    rng = np.random.default_rng(9)
    means = rng.normal(0.0, 0.15, size=(n, 3))
    log_scales = np.log(rng.uniform(0.25, 0.4, size=(n, 3)))
    quats = rng.normal(size=(n, 4))
    quats /= np.linalg.norm(quats, axis=-1, keepdims=True)
    logits = np.log(opacity / (1.0 - opacity)) + rng.normal(0.0, 0.1, size=n)
    sh = rng.normal(0.0, 0.05, size=(n, 16, 3))
    sh[:, 0] = rng.normal(0.5, 0.1, size=(n, 3))
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    params = scenes.SceneParams(f(means), f(log_scales), f(quats), f(logits), f(sh), 3)
    cam = scenes.orbit_cameras(1, 32, 24, 60.0, radius=3.0, seed=4)[0]
    sel = torch.arange(n) % 2 == 0
    for mode in ("gof", "radegs"):
        settings = RasterSettings(mode=mode, distortions="l1")
        ups = _ups(cam, 21)
        got, ggrads, out = run_gpu(params, cam, settings, sel, ups)
        most = out["stats"]["l1_max_samples"]
        assert lo <= most <= hi, most
        want, wgrads, _ = run_oracle(params, cam, mode, "l1", sel, ups)
        assert_images(got, want, mode, f"long/{mode}")
        assert_grads(ggrads, wgrads, f"long/{mode}")


def test_l1_exact_depth_ties_match_the_oracle():
    """Every fifth Gaussian of a surface-scene crop appears twice: the twins give
    bit-identical depths at every pixel, which the 32-bit key sort of the L1 resolve
    cannot tell apart, so those pixels take the 64-bit (depth, index) path.  Images
    must match; the twins' gradients are compared summed onto the original rows
    (a tie's order decides how dL1/ddepth splits between the twins, not its sum)."""
    torch.set_num_threads(8)
    params, cams = scenes.workload("surfaces100k_800", seed=0)
    n = params.means.shape[0]
    twin = torch.arange(0, n, 5)
    params = scenes.SceneParams(*(torch.cat((t, t[twin])) for t in params.tensors()), params.sh_degree)
    cam = cams[0].crop(384, 384, 48, 32)
    ups = _ups(cam, 31)
    for mode in ("gof", "radegs"):
        settings = RasterSettings(mode=mode, distortions="both")
        got, ggrads, _ = run_gpu(params, cam, settings, None, ups)
        want, wgrads, _ = run_oracle(params, cam, mode, "both", None, ups)
        assert_images(got, want, mode, f"ties/{mode}")
        for name in PARAM_NAMES + ("means2d_grad",):
            a, b = ggrads[name].clone(), wgrads[name].clone()
            a[twin] += a[n:]
            b[twin] += b[n:]
            e = rel_err(a[:n], b[:n])
            assert e < GRAD_RTOL, (mode, name, e)


def test_l1_wide_depth_span_matches_the_oracle():
    """Faint Gaussians strung along the viewing axis from depth 0.3 to 6: every pixel's
    samples span a depth ratio of 20, beyond what the resolve's packed 32-bit keys can
    hold, so those pixels take the 64-bit (depth, index) sort."""
    rng = np.random.default_rng(17)
    cam = scenes.orbit_cameras(1, 32, 24, 60.0, radius=3.0, seed=5)[0]
    origin = cam.origin.numpy().astype(np.float64)
    ahead = -origin / np.linalg.norm(origin)
    n = 90
    t = np.linspace(0.3, 6.0, n)
    means = origin[None] + t[:, None] * ahead[None] + rng.normal(0.0, 0.02, size=(n, 3))
    # anisotropic (an isotropic covariance has no quaternion gradient to compare)
    log_scales = np.log((0.08 * t + 0.2)[:, None] * rng.uniform(0.5, 1.5, size=(n, 3)))
    quats = rng.normal(size=(n, 4))
    quats /= np.linalg.norm(quats, axis=-1, keepdims=True)
    logits = np.log(0.05 / 0.95) + rng.normal(0.0, 0.1, size=n)
    sh = rng.normal(0.0, 0.05, size=(n, 16, 3))
    sh[:, 0] = rng.normal(0.5, 0.1, size=(n, 3))
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    params = scenes.SceneParams(f(means), f(log_scales), f(quats), f(logits), f(sh), 3)
    for mode in ("gof", "radegs"):
        settings = RasterSettings(mode=mode, distortions="both")
        ups = _ups(cam, 41)
        got, ggrads, out = run_gpu(params, cam, settings, None, ups)
        assert out["stats"]["l1_max_samples"] > 32
        want, wgrads, _ = run_oracle(params, cam, mode, "both", None, ups)
        assert_images(got, want, mode, f"span/{mode}")
        assert_grads(ggrads, wgrads, f"span/{mode}")


@pytest.mark.parametrize("mode", ["radegs", "gof", "ambisur"])
def test_render_settings_variants(mode):
    """The RenderConfig fields besides the mode: the antialiasing opacity compensation,
    a coloured background, a raised near plane and a lowered far plane that cut
    samples, a larger eps2d, and SH degrees below 3."""
    torch.set_num_threads(4)
    params, cams = scenes.workload("demo48", seed=0)
    sel = torch.arange(48) % 3 == 0
    variants = [
        dict(antialiased=True, background=(0.1, 0.5, 0.9), sh_degree=3),
        dict(near=2.6, far=3.4, eps2d=0.5, sh_degree=1),
        dict(antialiased=True, near=0.5, sh_degree=0),
        dict(background=(0.0, 0.0, 0.0), eps2d=0.1, sh_degree=2),
    ]
    for k, var in enumerate(variants):
        var = dict(var)
        degree = var.pop("sh_degree")
        p = scenes.SceneParams(params.means, params.log_scales, params.quats, params.opacity_logits,
                               params.sh, degree)
        gpu_settings = RasterSettings(mode=mode, distortions="both", **var)
        ora = oracle_render.RenderSettings(**var)
        for v in (0, 3, 6):
            cam = cams[v]
            ups = _ups(cam, 300 + 10 * k + v)
            got, ggrads, _ = run_gpu(p, cam, gpu_settings, sel, ups)
            want, wgrads, _ = run_oracle(p, cam, mode, "both", sel, ups, settings=ora)
            assert_images(got, want, mode, f"{mode}/variant{k}/v{v}")
            assert_grads(ggrads, wgrads, f"{mode}/variant{k}/v{v}")
