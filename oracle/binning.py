"""Exact tile lists in global stable depth order (TEST INFRASTRUCTURE).

Restates ``tile_members`` (src/splatforge/studio/tile_binning.py:10-34) with
vectorised numpy so that full-frame scenes of a million Gaussians finish in
seconds.  Arithmetic is float32 exactly as the reference performs it on its
float32 ``bounds`` array (``x - r`` in float32, divided by the tile size in
float32, then ``ceil``/``floor``; comparisons against ``near``/``far`` and the
image size in float32).

Returns CSR lists: ``offsets[T+1]`` and ``ids[I]`` (int64), tile-major,
row-major tiles, ids in stable depth order inside every tile.  ``keys`` gives
the 64-bit ``tile << 32 | float_bits(z)`` sort keys of that order.
"""

from __future__ import annotations

import math

import numpy as np


def tile_rects(bounds, *, width, height, tile_size, near, far):
    """Per-Gaussian inclusive tile rectangle and the keep mask (tile_binning.py:27-40)."""
    b = np.asarray(bounds, dtype=np.float32)
    if not np.isfinite(b).all():
        raise FloatingPointError("non-finite projected bounds")
    x, y, r, z = b[:, 0], b[:, 1], b[:, 2], b[:, 3]
    cols, rows = math.ceil(width / tile_size), math.ceil(height / tile_size)
    f32 = np.float32
    keep = (
        (z > f32(near))
        & (z < f32(far))
        & ~(x + r < f32(0))
        & ~(y + r < f32(0))
        & ~(x - r > f32(width))
        & ~(y - r > f32(height))
    )
    ts = f32(tile_size)
    with np.errstate(over="ignore", invalid="ignore"):
        lo_x = np.ceil(((x - r) / ts).astype(np.float64)) - 1
        hi_x = np.floor(((x + r) / ts).astype(np.float64))
        lo_y = np.ceil(((y - r) / ts).astype(np.float64)) - 1
        hi_y = np.floor(((y + r) / ts).astype(np.float64))
    left = np.maximum(0, lo_x)
    right = np.minimum(cols - 1, hi_x)
    top = np.maximum(0, lo_y)
    bottom = np.minimum(rows - 1, hi_y)
    rect = np.stack((left, top, right, bottom), 1)
    rect = np.where(keep[:, None], rect, 0).astype(np.int64)
    count = np.where(
        keep, np.maximum(0, rect[:, 2] - rect[:, 0] + 1) * np.maximum(0, rect[:, 3] - rect[:, 1] + 1), 0
    )
    return rect, count, keep, cols, rows


def tile_lists(bounds, *, width, height, tile_size, near, far):
    rect, count, keep, cols, rows = tile_rects(
        bounds, width=width, height=height, tile_size=tile_size, near=near, far=far
    )
    z = np.asarray(bounds, dtype=np.float32)[:, 3]
    order = np.argsort(z, kind="stable")
    order = order[count[order] > 0]
    cnt = count[order]
    total = int(cnt.sum())
    gid = np.repeat(order, cnt)
    start = np.repeat(np.cumsum(cnt) - cnt, cnt)
    local = np.arange(total, dtype=np.int64) - start
    r = rect[gid]
    w = r[:, 2] - r[:, 0] + 1
    tx = r[:, 0] + local % w
    ty = r[:, 1] + local // w
    tile = ty * cols + tx
    perm = np.argsort(tile, kind="stable")
    ids = gid[perm]
    tiles = tile[perm]
    offsets = np.zeros(cols * rows + 1, dtype=np.int64)
    np.add.at(offsets, tiles + 1, 1)
    offsets = np.cumsum(offsets)
    zbits = z.view(np.uint32).astype(np.uint64)
    keys = (tiles.astype(np.uint64) << np.uint64(32)) | zbits[ids]
    return offsets, ids.astype(np.int64), keys


def as_members(offsets, ids):
    """CSR -> the reference's list-of-arrays form."""
    return [ids[offsets[t] : offsets[t + 1]] for t in range(len(offsets) - 1)]
