"""sf_b200_bin_order_static against sf_b200_bin_order, through the C ABI.

The static variant is for callers that may not allocate device memory (their host
application owns the device budget); it works in a scratch array compiled into the
library.  Its depth order and intersection offsets must equal the allocating entry
point's exactly (integer results), on two calls in a row -- the second call finds
the first call's leftovers in the shared array.

This file is collected last on purpose: if it fails, a run that stops at the first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from splatforge_b200 import _lib
from splatforge_b200.rasterizer import _ptr, _stream

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(n, seed):
    g = torch.Generator().manual_seed(seed)
    count = torch.randint(0, 40, (n,), generator=g, dtype=torch.int32)
    count[torch.rand(n, generator=g) < 0.2] = 0  # culled Gaussians
    z = torch.rand(n, generator=g) * 8 + 0.5
    z[: n // 7] = z[n // 7 : 2 * (n // 7)]  # exact depth ties (stable order by index)
    key = z.view(torch.int32).clone()
    key[count == 0] = -1  # 0xffffffff for culled
    return count.to(DEV), key.to(DEV)


def _with_workspace(count, key):
    n = count.shape[0]
    size = ctypes.c_size_t()
    _lib.call("sf_b200_bin_workspace_bytes", n, 0, 1, ctypes.byref(size))
    ws = torch.empty((max(size.value, 1),), device=DEV, dtype=torch.uint8)
    order = torch.empty((n,), device=DEV, dtype=torch.int32)
    offsets = torch.empty((n + 1,), device=DEV, dtype=torch.int64)
    _lib.call("sf_b200_bin_order", _ptr(count), _ptr(key), n, _ptr(order), _ptr(offsets), _ptr(ws),
              size.value, _stream(torch.device(DEV)))
    return order.cpu().numpy(), offsets.cpu().numpy()


def _static(count, key):
    n = count.shape[0]
    order = torch.full((n,), -7, device=DEV, dtype=torch.int32)
    offsets = torch.full((n + 1,), -7, device=DEV, dtype=torch.int64)
    _lib.call("sf_b200_bin_order_static", _ptr(count), _ptr(key), n, _ptr(order), _ptr(offsets),
              _stream(torch.device(DEV)))
    return order.cpu().numpy(), offsets.cpu().numpy()


def test_static_scratch_matches_allocating_entry_point_twice():
    for n, seed in ((1 << 20, 1), (300_001, 2)):  # the maximum size, then a smaller call
        count, key = _inputs(n, seed)
        want = _with_workspace(count, key)
        got = _static(count, key)
        np.testing.assert_array_equal(got[0], want[0])
        np.testing.assert_array_equal(got[1], want[1])
        torch.cuda.synchronize()


def test_static_scratch_call_allocates_no_device_memory():
    """After a first call (which resolves the array's address), a call changes neither
    the device's free memory nor torch's allocated bytes."""
    n = 1 << 20
    count, key = _inputs(n, 3)
    order = torch.empty((n,), device=DEV, dtype=torch.int32)
    offsets = torch.empty((n + 1,), device=DEV, dtype=torch.int64)
    stream = _stream(torch.device(DEV))

    def call():
        _lib.call("sf_b200_bin_order_static", _ptr(count), _ptr(key), n, _ptr(order), _ptr(offsets), stream)

    call()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_static_scratch_rejects_oversized_input():
    n = (1 << 20) + 1
    count = torch.zeros((n,), device=DEV, dtype=torch.int32)
    key = torch.zeros((n,), device=DEV, dtype=torch.int32)
    with pytest.raises(_lib.NativeError, match="1048576"):
        _static(count, key)
