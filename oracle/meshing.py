"""GOF mesh extraction restated on the CPU (TEST INFRASTRUCTURE; see ``oracle/__init__.py``).

* ``grid(...)``                 -- the exporter's tetrahedral grid
                                   (src/splatforge/studio/exporters.py:20-38);
* ``triangulate(points, radii)`` -- Delaunay cells with the radius filter
                                   (src/splatforge/mesh/tetrahedra.py:19-31);
* ``marching_tetrahedra(...)``  -- shared-edge bisection and oriented faces
                                   (src/splatforge/mesh/tetrahedra.py:34-109).

The marching step is written as a per-mask table rather than the reference's per-cell
loop; each table entry follows the reference's rule for that split (pivot vertex for
1/3 splits, the two-triangle quad for 2/2 splits).  Float64 expressions are evaluated
in the reference's order, so equal field values give equal vertices and faces.
Delaunay triangulation uses scipy's Qhull binding, as the reference does.
"""

from __future__ import annotations

import numpy as np
from scipy.spatial import Delaunay

EDGE_A = np.array([0, 0, 0, 1, 1, 2])
EDGE_B = np.array([1, 2, 3, 2, 3, 3])


def _edge(a, b):
    a, b = min(a, b), max(a, b)
    return {(0, 1): 0, (0, 2): 1, (0, 3): 2, (1, 2): 3, (1, 3): 4, (2, 3): 5}[(a, b)]


def _mask_table():
    """For every inside-mask (bit k = vertex k inside): the faces as edge indices, the
    inside vertices and the outside vertices (ascending local order)."""
    table = {}
    for m in range(1, 15):
        inn = [k for k in range(4) if (m >> k) & 1]
        out = [k for k in range(4) if not (m >> k) & 1]
        if len(inn) in (1, 3):
            pivot = inn[0] if len(inn) == 1 else out[0]
            rest = out if len(inn) == 1 else inn
            faces = [[_edge(pivot, r) for r in rest]]
        else:
            (a, b), (c, d) = inn, out
            faces = [[_edge(a, c), _edge(a, d), _edge(b, c)], [_edge(a, d), _edge(b, d), _edge(b, c)]]
        table[m] = (np.array(faces), inn, out)
    return table


_TABLE = _mask_table()


def triangulate(points, radii=None):
    """Delaunay tetrahedra, keeping only cells whose six edges are no longer than the sum
    of their end points' radii (+1e-10) when radii are given (tetrahedra.py:19-31)."""
    points = np.asarray(points, np.float64)
    if len(points) < 4 or np.linalg.matrix_rank(points - points.mean(0)) < 3:
        raise ValueError("tetrahedral extraction needs >=4 noncoplanar points")
    cells = Delaunay(points).simplices.astype(np.int64)
    if radii is None:
        return cells
    radii = np.asarray(radii)
    a, b = cells[:, EDGE_A], cells[:, EDGE_B]
    length = np.linalg.norm(points[a] - points[b], axis=-1)
    return cells[(length <= radii[a] + radii[b] + 1e-10).all(-1)]


def grid(means, quats, scales, opacities, *, seed_opacity_min=0.05, max_gaussians=None, tetra_extent=3.0):
    """(unique points [U,3] float64, vertex radii [U], seed count) of exporters.py:20-38.
    Inputs are float32 numpy arrays of the activated scene (scales exponentiated,
    opacities after the sigmoid)."""
    opacities = np.asarray(opacities, np.float32)
    seeds = np.flatnonzero(opacities >= seed_opacity_min)
    if not len(seeds):
        raise ValueError("no Gaussian passes the mesh seed opacity threshold")
    if max_gaussians is not None and len(seeds) > max_gaussians:
        seeds = seeds[np.argsort(opacities[seeds])[-max_gaussians:]]
    q = np.asarray(quats, np.float32)[seeds]
    s = np.asarray(scales, np.float32)[seeds]
    m = np.asarray(means, np.float32)[seeds]
    R = _rotations(q)
    signs = np.zeros((9, 3))
    signs[1:] = [[x, y, z] for x in (-1.0, 1.0) for y in (-1.0, 1.0) for z in (-1.0, 1.0)]
    local = signs[None] * s[:, None].astype(np.float64) * tetra_extent          # [n, 9, 3]
    Rd = R.astype(np.float64)
    # (R_r0 l0 + R_r1 l1) + R_r2 l2 for every row r
    rot = (Rd[:, None, :, 0] * local[:, :, None, 0] + Rd[:, None, :, 1] * local[:, :, None, 1]) \
        + Rd[:, None, :, 2] * local[:, :, None, 2]
    pts = (m[:, None].astype(np.float64) + rot).reshape(-1, 3)
    unique, inverse = np.unique(pts, axis=0, return_inverse=True)
    radius = np.zeros(len(unique))
    np.maximum.at(radius, inverse.reshape(-1), np.repeat(s.max(-1) * np.float32(tetra_extent), 9))
    return unique, radius, len(seeds)


def _rotations(q):
    """float32 wxyz -> R after normalisation, evaluated in float32 (reference.py:15-30)."""
    n = np.sqrt((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2] + q[:, 3] * q[:, 3])
    q = q / np.maximum(n, np.float32(1e-12))[:, None]
    w, x, y, z = q.T
    one, two = np.float32(1), np.float32(2)
    rows = (one - two * (y * y + z * z), two * (x * y - w * z), two * (x * z + w * y),
            two * (x * y + w * z), one - two * (x * x + z * z), two * (y * z - w * x),
            two * (x * z - w * y), two * (y * z + w * x), one - two * (x * x + y * y))
    return np.stack(rows, -1).reshape(-1, 3, 3).astype(np.float32)


def marching_tetrahedra(points, cells, values, field, *, level=0.0, binary_steps=8, inside_greater=True):
    """(vertices [U,3] float64, faces [F,3] int64): one vertex per crossing edge (in
    ascending (low, high) vertex order) after ``binary_steps`` bisections against
    ``field`` (float64 [M,3] -> [M]), faces in cell order oriented away from the inside
    vertices, faces with area <= 1e-16 removed (tetrahedra.py:34-109)."""
    points = np.asarray(points, np.float64)
    cells = np.asarray(cells, np.int64)
    values = np.asarray(values, np.float64)
    if values.shape != (len(points),) or not np.isfinite(values).all():
        raise ValueError("field returned invalid vertex scalars")
    inside = values >= level if inside_greater else values <= level
    mask = inside[cells].astype(np.int64) @ np.array([1, 2, 4, 8]) if len(cells) else np.zeros(0, np.int64)
    act = (mask != 0) & (mask != 15)
    cells, mask = cells[act], mask[act]
    if not len(cells):
        return np.empty((0, 3)), np.empty((0, 3), np.int64)
    ins = inside[cells]
    crossing = ins[:, EDGE_A] != ins[:, EDGE_B]
    va, vb = cells[:, EDGE_A], cells[:, EDGE_B]
    pairs = np.stack([np.minimum(va, vb)[crossing], np.maximum(va, vb)[crossing]], -1)
    edges, inverse = np.unique(pairs, axis=0, return_inverse=True)
    low, high = points[edges[:, 0]].copy(), points[edges[:, 1]].copy()
    low_in = inside[edges[:, 0]]
    for _ in range(binary_steps):
        mid = (low + high) / 2
        v = np.asarray(field(mid))
        if v.shape != (len(mid),) or not np.isfinite(v).all():
            raise ValueError("field returned invalid bisection scalars")
        same = (v >= level if inside_greater else v <= level) == low_in
        low[same] = mid[same]
        high[~same] = mid[~same]
    vertices = (low + high) / 2
    row = np.full(crossing.shape, -1, np.int64)
    row[crossing] = inverse.reshape(-1)

    n_faces = np.where(np.isin(mask, [3, 5, 6, 9, 10, 12]), 2, 1)
    start = np.concatenate(([0], np.cumsum(n_faces)[:-1]))
    faces = np.empty((int(n_faces.sum()), 3), np.int64)
    outward_of = np.empty((len(faces), 3))
    for m, (tri, inn, out) in _TABLE.items():
        sel = np.flatnonzero(mask == m)
        if not len(sel):
            continue
        so = points[cells[sel, out[0]]]
        for k in out[1:]:
            so = so + points[cells[sel, k]]
        si = points[cells[sel, inn[0]]]
        for k in inn[1:]:
            si = si + points[cells[sel, k]]
        outward = so / len(out) - si / len(inn)
        for t in range(len(tri)):
            faces[start[sel] + t] = row[sel][:, tri[t]]
            outward_of[start[sel] + t] = outward
    v0, v1, v2 = (vertices[faces[:, k]] for k in range(3))
    c = _cross(v1 - v0, v2 - v0)
    flip = (c[:, 0] * outward_of[:, 0] + c[:, 1] * outward_of[:, 1]) + c[:, 2] * outward_of[:, 2] < 0
    faces[flip, 1], faces[flip, 2] = faces[flip, 2].copy(), faces[flip, 1].copy()
    area = np.sqrt((c[:, 0] * c[:, 0] + c[:, 1] * c[:, 1]) + c[:, 2] * c[:, 2])
    return vertices, faces[area > 1e-16]


def _cross(a, b):
    return np.stack([a[:, 1] * b[:, 2] - a[:, 2] * b[:, 1],
                     a[:, 2] * b[:, 0] - a[:, 0] * b[:, 2],
                     a[:, 0] * b[:, 1] - a[:, 1] * b[:, 0]], -1)
