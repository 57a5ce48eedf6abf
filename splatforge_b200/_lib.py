"""ctypes binding of ``libsf_b200.so`` (the C ABI in include/splatforge_b200.h).

Loading fails loudly when the library is missing: there is no CPU or Torch fallback
anywhere in this package.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_float, c_int32, c_int64, c_size_t, c_uint8, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libsf_b200.so"

SF_OK = 0
SF_ERR_CAPACITY = 3
MODE = {"radegs": 0, "gof": 1, "ambisur": 2}
DISTORTIONS = {"none": 0, "l1": 1, "l2": 2, "both": 3}
RECORD_FLOATS = 20
PIXEL_STATE_FLOATS = 16
L1_SAMPLE_FLOATS = 2


class Camera(ctypes.Structure):
    _fields_ = [
        ("R", c_float * 9),
        ("t", c_float * 3),
        ("K", c_float * 9),
        ("Kinv", c_float * 9),
        ("origin", c_float * 3),
        ("width", c_int32),
        ("height", c_int32),
    ]


class Settings(ctypes.Structure):
    _fields_ = [
        ("mode", c_int32),
        ("distortions", c_int32),
        ("tile_size", c_int32),
        ("sh_degree", c_int32),
        ("sh_coeffs", c_int32),
        ("antialiased", c_int32),
        ("extent", c_float),
        ("extent_sq", c_float),
        ("eps2d", c_float),
        ("near_plane", c_float),
        ("far_plane", c_float),
        ("background", c_float * 3),
        ("t_stop", c_float),
    ]


P = c_void_p  # every device pointer travels as an untyped address
_SIGNATURES = {
    "sf_b200_last_error": (ctypes.c_char_p, []),
    "sf_b200_abi_version": (ctypes.c_int, []),
    "sf_b200_kernel_launches": (ctypes.c_int64, []),
    "sf_b200_covariance_forward": (ctypes.c_int, [P, P, c_int64, P, P]),
    "sf_b200_covariance_backward": (ctypes.c_int, [P, P, c_int64, P, P, P, P]),
    "sf_b200_sh_color_forward": (ctypes.c_int, [P, c_int32, P, c_int64, c_int32, P, P]),
    "sf_b200_sh_color_backward": (ctypes.c_int, [P, c_int32, P, c_int64, c_int32, P, P, P, P]),
    "sf_b200_project_forward": (
        ctypes.c_int,
        [P, P, P, P, P, P, c_int64, POINTER(Camera), POINTER(Settings), P, P, P, P, P, P, P, P],
    ),
    "sf_b200_project_backward": (
        ctypes.c_int,
        [P, P, P, P, P, c_int64, POINTER(Camera), POINTER(Settings), P, P, P, P, P, P, P, P],
    ),
    "sf_b200_bin_rects": (
        ctypes.c_int,
        [P, c_int64, c_int32, c_int32, c_int32, c_float, c_float, P, P, P, P, P],
    ),
    "sf_b200_bin_workspace_bytes": (ctypes.c_int, [c_int64, c_int64, c_int32, POINTER(c_size_t)]),
    "sf_b200_bin_order": (ctypes.c_int, [P, P, c_int64, P, P, P, c_size_t, P]),
    "sf_b200_bin_emit": (
        ctypes.c_int,
        [P, P, P, c_int64, c_int64, c_int32, c_int32, P, P, P, c_size_t, P],
    ),
    "sf_b200_bin_emit_bounded": (
        ctypes.c_int,
        [P, P, P, c_int64, c_int64, c_int32, c_int32, P, P, P, c_size_t, P, P],
    ),
    "sf_b200_bin_keys": (ctypes.c_int, [P, P, P, c_int32, c_int64, P, P]),
    "sf_b200_bin_order_static": (ctypes.c_int, [P, P, c_int64, P, P, P]),
    "sf_b200_opacity_field_workspace_bytes": (ctypes.c_int, [c_int64, POINTER(c_size_t)]),
    "sf_b200_opacity_field": (ctypes.c_int, [P, c_int64, P, P, P, c_int64, P, c_int32, P, P, c_size_t, P]),
    "sf_b200_composite_workspace_bytes": (ctypes.c_int, [c_int64, c_int64, c_int64, c_int32, POINTER(c_size_t)]),
    "sf_b200_alpha_composite_forward": (
        ctypes.c_int,
        [P, P, P, P, c_int64, c_int64, c_int64, c_int32] + [P] * 8 + [P, c_size_t, P],
    ),
    "sf_b200_alpha_composite_backward": (
        ctypes.c_int,
        [P, P, P, P, c_int64, c_int64, c_int64, c_int32, P, P, c_size_t] + [P] * 8 + [P] * 4 + [P],
    ),
    "sf_b200_opacity_field_culled_workspace_bytes": (
        ctypes.c_int, [c_int64, c_int64, c_int64, c_int32, POINTER(c_size_t)]
    ),
    "sf_b200_opacity_field_culled": (
        ctypes.c_int,
        [P, c_int64, P, P, P, c_int64, P, c_int32, c_float, c_int32, P, P, c_size_t, c_int64, POINTER(c_int64), P],
    ),
    "sf_b200_opacity_field_culled_stats": (
        ctypes.c_int,
        [P, c_int64, P, P, P, c_int64, P, c_int32, c_float, c_int32, P, P, c_size_t, c_int64, POINTER(c_int64), P,
         POINTER(c_float), P],
    ),
    "sf_b200_opacity_field_plan_bytes": (ctypes.c_int, [c_int64, c_int32, c_int32, c_int64, c_int64, POINTER(c_size_t)]),
    "sf_b200_opacity_field_plan_build": (
        ctypes.c_int, [P, P, P, c_int64, P, c_int32, c_float, c_int32, P, c_size_t, c_int64, c_int64, P, P]
    ),
    "sf_b200_opacity_field_plan_query_bytes": (ctypes.c_int, [c_int64, c_int32, c_int32, POINTER(c_size_t)]),
    "sf_b200_opacity_field_plan_eval": (
        ctypes.c_int, [P, c_int64, c_int32, c_int32, c_int64, c_int64, P, P, c_int64, P, P, c_size_t, P]
    ),
    "sf_b200_pixel_rays": (ctypes.c_int, [P, c_int32, c_int32, P, P]),
    "sf_b200_ray_peak": (ctypes.c_int, [P, P, c_int64, P, P, c_int64, P, P, P, P]),
    "sf_b200_depth_normals": (ctypes.c_int, [P, P, c_int32, c_int32, P, P, P]),
    "sf_b200_depth_normals_backward": (ctypes.c_int, [P, P, c_int32, c_int32, P, P, P, P]),
    "sf_b200_sh_ambiguity": (ctypes.c_int, [P, c_int64, c_int32, P, P]),
    "sf_b200_sh_ambiguity_backward": (ctypes.c_int, [P, c_int64, c_int32, P, P, P]),
    "sf_b200_ray_color_variance": (ctypes.c_int, [P, P, P, c_int64, c_int64, c_int64, P, P]),
    "sf_b200_ray_color_variance_backward": (ctypes.c_int, [P, P, P, P, c_int64, c_int64, c_int64, P, P]),
    "sf_b200_patch_zncc": (ctypes.c_int, [P, P, P, c_int64, c_int32, c_float, P, P, P]),
    "sf_b200_patch_zncc_backward": (ctypes.c_int, [P, P, P, c_int64, c_int32, c_float, P, P, P, P]),
    "sf_b200_densify_observe": (ctypes.c_int, [P, P, c_int64, c_float, c_float, P, P, P]),
    "sf_b200_normal_consistency_workspace_bytes": (ctypes.c_int, [c_int32, c_int32, POINTER(c_size_t)]),
    "sf_b200_normal_consistency": (ctypes.c_int, [P, P, c_int32, c_int32, P, P, P, P, P, P, P, c_size_t, P]),
    "sf_b200_normal_consistency_backward": (
        ctypes.c_int, [P, P, c_int32, c_int32, P, P, P, P, P, P, P, P, P, P, P, c_size_t, P]
    ),
    "sf_b200_mesh_grid_points": (ctypes.c_int, [P, P, P, P, c_int64, c_double, P, P, P]),
    "sf_b200_mesh_count_workspace_bytes": (ctypes.c_int, [c_int64, POINTER(c_size_t)]),
    "sf_b200_mesh_count": (ctypes.c_int, [P, c_int64, P, c_int64, c_double, c_int32, P, P, P, P, c_size_t, P]),
    "sf_b200_mesh_edges_workspace_bytes": (ctypes.c_int, [c_int64, POINTER(c_size_t)]),
    "sf_b200_mesh_edges": (
        ctypes.c_int, [P, c_int64, P, c_int64, P, P, c_int64, P, P, P, P, P, P, P, c_size_t, P]
    ),
    "sf_b200_mesh_midpoints": (ctypes.c_int, [P, P, c_int64, P, P]),
    "sf_b200_mesh_bisect": (ctypes.c_int, [P, P, P, c_int64, P, c_double, c_int32, P]),
    "sf_b200_mesh_faces_workspace_bytes": (ctypes.c_int, [c_int64, POINTER(c_size_t)]),
    "sf_b200_mesh_faces": (
        ctypes.c_int, [P, P, c_int64, P, P, P, P, P, c_int64, P, c_int64, P, P, P, P, c_size_t, P]
    ),
    "sf_b200_raster_forward": (
        ctypes.c_int,
        [P, c_int64, P, P, POINTER(Camera), POINTER(Settings)]
        + [P] * 10
        + [P, c_int64, P, c_int32, P, P, P],
    ),
    "sf_b200_l1_offsets": (ctypes.c_int, [POINTER(Camera), P, P, P, c_size_t, P]),
    "sf_b200_l1_resolve": (
        ctypes.c_int,
        [POINTER(Camera), POINTER(Settings), P, P, c_int64, P, c_int32, c_int32, P, P],
    ),
    "sf_b200_raster_backward": (
        ctypes.c_int,
        [P, c_int64, P, P, POINTER(Camera), POINTER(Settings), P, P, c_int64, P, c_int32]
        + [P] * 9
        + [P, P, P, P, P],
    ),
}

_lib = None


class NativeError(RuntimeError):
    """A non-zero status from libsf_b200 (message from sf_b200_last_error)."""


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m splatforge_b200.build` "
                "(the B200 provider has no CPU fallback)"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.sf_b200_abi_version() != 1:
            raise ImportError("libsf_b200.so ABI version mismatch")
        _lib = handle
    return _lib


def call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != SF_OK:
        msg = lib().sf_b200_last_error().decode(errors="replace")
        if rc == 1:
            raise ValueError(f"{name}: {msg}")
        raise NativeError(f"{name} failed ({rc}): {msg}")


def declared_symbols():
    return sorted(_SIGNATURES)
