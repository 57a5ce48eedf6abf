"""The C ABI library loads, exports every declared entry point and validates its
arguments before touching a device (CPU only; no compute calls)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from splatforge_b200 import _lib, build

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "splatforge_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(sf_b200_\w+)\s*\(", text)))


def test_library_builds_and_exports_every_declared_symbol():
    lib_path = build.build_library()
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (sf_b200_\w+)", out.stdout))
    missing = [s for s in declared() if s not in exported]
    assert not missing, missing
    # the ctypes binding covers the same set
    assert set(_lib.declared_symbols()) == set(declared())


def test_abi_version_and_error_paths_without_a_device():
    lib = _lib.lib()
    assert lib.sf_b200_abi_version() == 1
    cam = _lib.Camera()
    cam.width, cam.height = 32, 32
    st = _lib.Settings()
    st.mode = 7  # invalid
    st.tile_size = 16
    st.extent = 3.0
    rc = lib.sf_b200_project_forward(*([None] * 6), 1, ctypes.byref(cam), ctypes.byref(st), *([None] * 7), None)
    assert rc == 1
    assert b"rendering mode" in lib.sf_b200_last_error()
    st.mode = 1
    st.tile_size = 8
    rc = lib.sf_b200_project_forward(*([None] * 6), 1, ctypes.byref(cam), ctypes.byref(st), *([None] * 7), None)
    assert rc == 1 and b"tile_size" in lib.sf_b200_last_error()
    size = ctypes.c_size_t()
    assert lib.sf_b200_bin_workspace_bytes(1000, 5000, 64, ctypes.byref(size)) == 0
    assert size.value > 0
    assert lib.sf_b200_bin_workspace_bytes(1000, 1 << 33, 64, ctypes.byref(size)) == 3
    with pytest.raises(ValueError):
        _lib.call("sf_b200_sh_color_forward", None, 4, None, 10, 7, None, None)
    # the bounded emit refuses a missing overflow flag or a capacity of zero before any launch
    rc = lib.sf_b200_bin_emit_bounded(None, None, None, 10, 1000, 4, 16, None, None, None, 0, None, None)
    assert rc == 1 and b"bin_emit_bounded" in lib.sf_b200_last_error()
    rc = lib.sf_b200_bin_emit_bounded(None, None, None, 10, 0, 4, 16, None, None, None, 0, None, None)
    assert rc == 1


def test_size_classes_and_intersection_capacity():
    from splatforge_b200 import rasterizer

    seen = set()
    for n in range(1, 1 << 24, 99991):
        c = rasterizer._size_class(n)
        assert n <= c <= max(n, int(n * 1.125) + 1)
        seen.add(c)
    assert len(seen) < ((1 << 24) // 99991) // 3  # few distinct sizes
    for total in (0, 5000, 52_349_663):
        cap = rasterizer._isect_capacity(total)
        assert cap >= 1.2 * total and cap == rasterizer._size_class(cap)


def test_rasterize_rejects_cpu_tensors_without_fallback():
    import torch

    from splatforge_b200 import scenes
    from splatforge_b200.rasterizer import RasterSettings, rasterize

    params, cams = scenes.workload("demo48", seed=0)
    v = scenes.activated(params)
    with pytest.raises(ValueError, match="no CPU fallback"):
        rasterize(v.means, v.quats, v.scales, v.opacities, v.sh, 3, cams[0], RasterSettings())
    with pytest.raises(ValueError):
        RasterSettings(mode="splat").struct(3, 16)
    with pytest.raises(ValueError):
        RasterSettings(distortions="l3").struct(3, 16)
    del torch


def test_static_scratch_covers_the_ordering_workspace_at_its_limit():
    """The static array behind sf_b200_bin_order_static holds the ordering workspace of
    the largest call it accepts (host arithmetic only, no device)."""
    text = HEADER.read_text()
    limit = int(re.search(r"#define SF_B200_STATIC_MAX_GAUSSIANS (\d+)", text).group(1))
    m = re.search(r"#define SF_B200_STATIC_SCRATCH_BYTES \((\d+)u << (\d+)\)", text)
    scratch = int(m.group(1)) << int(m.group(2))
    size = ctypes.c_size_t()
    assert _lib.lib().sf_b200_bin_workspace_bytes(limit, 0, 1, ctypes.byref(size)) == 0
    assert size.value <= scratch, (size.value, scratch)
