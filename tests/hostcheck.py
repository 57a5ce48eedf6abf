"""CPU driver of libsf_b200_hostcheck.so: the kernels' arithmetic, sequential.

Runs the same projection / tile evaluation / reverse-mode functions the CUDA kernels
call (splatforge_b200/csrc/sf_math.cuh, sf_grad.cuh) on CPU tensors, with the
oracle's tile lists, so the hand-written gradients can be checked against autograd
of the oracle without a GPU.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle import binning
from splatforge_b200 import build
from splatforge_b200._lib import L1_SAMPLE_FLOATS, PIXEL_STATE_FLOATS, RECORD_FLOATS, Camera, Settings
from splatforge_b200.rasterizer import camera_struct

_hc = None


def lib():
    global _hc
    if _hc is None:
        path = build.build_hostcheck()
        h = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        h.hc_project_forward.argtypes = [P] * 6 + [ctypes.c_int64, ctypes.POINTER(Camera), ctypes.POINTER(Settings)] + [P] * 6
        h.hc_project_backward.argtypes = [P] * 5 + [ctypes.c_int64, ctypes.POINTER(Camera), ctypes.POINTER(Settings)] + [P] * 7
        h.hc_raster_forward.argtypes = [P, P, P, ctypes.POINTER(Camera), ctypes.POINTER(Settings)] + [P] * 11 + [ctypes.c_int64, ctypes.c_int32]
        h.hc_raster_backward.argtypes = [P, ctypes.c_int64, P, P, ctypes.POINTER(Camera), ctypes.POINTER(Settings), P, P, ctypes.c_int64, ctypes.c_int32] + [P] * 12
        F = ctypes.c_float
        h.hc_box_may_pass.argtypes = [P, ctypes.c_int64, F, F, F, F, F, P]
        _hc = h
    return _hc


def box_may_pass(gauss, box, ext2):
    """The kernels' warp-culling predicate for [n, 5] (qa, qb, qc, X, Y) float32 rows."""
    g = torch.as_tensor(gauss, dtype=torch.float32).contiguous()
    out = torch.zeros(g.shape[0], dtype=torch.uint8)
    lib().hc_box_may_pass(_p(g), g.shape[0], *(ctypes.c_float(v) for v in box), ctypes.c_float(ext2), _p(out))
    return out.bool().numpy()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


CH = (("rgb", 3), ("alpha", 1), ("depth", 1), ("normals", 3), ("distortion_l1", 1),
      ("distortion_l2", 1), ("median_depth", 1), ("ray_color", 1), ("ambiguity_mask", 1))


def render(params, camera, settings, *, selected=None, ups=None, cap=None):
    """Forward (+ backward when ``ups`` is given) through the host-compiled kernels.

    Returns (images dict, grads dict or None, extras)."""
    h = lib()
    means = params.means.contiguous()
    quats = params.quats.contiguous()
    scales = params.log_scales.exp().contiguous()
    opac = params.opacity_logits.sigmoid().contiguous()
    sh = params.sh.contiguous()
    n = means.shape[0]
    cam = camera_struct(camera)
    st = settings.struct(params.sh_degree, sh.shape[1])
    sel = None if selected is None else selected.to(torch.uint8).contiguous()
    means2d = torch.empty(n, 2)
    radii = torch.empty(n)
    records = torch.empty(n, RECORD_FLOATS)
    rect = torch.empty(n, 4, dtype=torch.int32)
    count = torch.empty(n, dtype=torch.int32)
    dkey = torch.empty(n, dtype=torch.int32)
    h.hc_project_forward(_p(means), _p(quats), _p(scales), _p(opac), _p(sh), _p(sel), n,
                         ctypes.byref(cam), ctypes.byref(st), _p(means2d), _p(radii), _p(records),
                         _p(rect), _p(count), _p(dkey))
    z = records[:, 10]
    bounds = torch.stack((means2d[:, 0], means2d[:, 1], radii, z), 1).numpy()
    offsets, ids, _ = binning.tile_lists(bounds, width=camera.width, height=camera.height, tile_size=16,
                                         near=settings.near, far=settings.far)
    ids_t = torch.from_numpy(ids.astype(np.int32))
    ranges = torch.from_numpy(np.stack((offsets[:-1], offsets[1:]), 1).astype(np.int32)).contiguous()
    H, W = camera.height, camera.width
    imgs = {name: torch.zeros(H, W, c) for name, c in CH}
    state = torch.zeros(H * W, PIXEL_STATE_FLOATS)
    T = ranges.shape[0]
    if cap is None:
        cap = int(max(1, (offsets[1:] - offsets[:-1]).max(initial=1)))
    slots = T * cap * 256
    l1s = torch.zeros(L1_SAMPLE_FLOATS, slots) if (st.distortions & 1) else torch.zeros(1)
    h.hc_raster_forward(_p(records), _p(ids_t), _p(ranges), ctypes.byref(cam), ctypes.byref(st),
                        *(_p(imgs[name]) for name, _ in CH), _p(state), _p(l1s), slots, cap)
    extras = {"means2d": means2d, "radii": radii, "records": records, "state": state, "ids": ids_t, "l1s": l1s, "cap": cap,
              "ranges": ranges}
    if ups is None:
        return imgs, None, extras
    g_rec = torch.zeros(n, RECORD_FLOATS)
    g_xy = torch.zeros(n, 2)
    absgrad = torch.zeros(n, 2)
    upl = [ups[name].contiguous() for name, _ in CH]
    h.hc_raster_backward(_p(records), n, _p(ids_t), _p(ranges), ctypes.byref(cam), ctypes.byref(st), _p(state),
                         _p(l1s), slots, cap, *(_p(u) for u in upl), _p(g_rec), _p(g_xy), _p(absgrad))
    gm, gq, gs, go, gsh = (torch.zeros_like(t) for t in (means, quats, scales, opac, sh))
    h.hc_project_backward(_p(means), _p(quats), _p(scales), _p(opac), _p(sh), n, ctypes.byref(cam),
                          ctypes.byref(st), _p(g_xy), _p(g_rec), _p(gm), _p(gq), _p(gs), _p(go), _p(gsh))
    grads = {
        "means": gm,
        "log_scales": gs * scales,
        "quats": gq,
        "opacity_logits": go * opac * (1 - opac),
        "sh": gsh,
        "means2d_grad": g_xy,
        "absgrad": absgrad,
    }
    return imgs, grads, extras
