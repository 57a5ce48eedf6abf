"""GOF mesh extraction with the marching stages on the device.

SplatForge's GOF exporter (src/splatforge/studio/exporters.py:20-102) builds a
tetrahedral grid on the seed Gaussians' centres and extent-sigma box corners, evaluates
the opacity field at every grid point, extracts the field's level set with marching
tetrahedra and shared-edge bisection (src/splatforge/mesh/tetrahedra.py:34-109), and
writes a PLY mesh.  Here:

* on the device (libsf_b200.so): the grid points (``sf_b200_mesh_grid_points``), the
  opacity field (a culled ``ops.OpacityFieldPlan``, or the brute-force ``ops.opacity_field``)
  and every marching stage (``sf_b200_mesh_count`` / ``_edges`` / ``_midpoints`` /
  ``_bisect`` / ``_faces``): inside flags, active cells, crossing-edge deduplication, the
  bisection updates and the oriented faces;
* on the host, as in the reference: deduplication of the grid points and the Delaunay
  triangulation (scipy's Qhull binding) with its radius filter.

With equal field values the vertices and faces are the reference's, bit for bit (the
float64 expressions use explicitly rounded operations in the reference's order).
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

from . import ops
from ._lib import call
from .rasterizer import _ptr, _stream

EDGE_A = np.array([0, 0, 0, 1, 1, 2])
EDGE_B = np.array([1, 2, 3, 2, 3, 3])


def _device_of(*items):
    for t in items:
        if isinstance(t, torch.Tensor) and t.device.type == "cuda":
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("mesh extraction runs on a CUDA device (no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _workspace(query, n, dev):
    size = ctypes.c_size_t()
    call(query, int(n), ctypes.byref(size))
    return torch.empty((max(size.value, 1),), dtype=torch.uint8, device=dev)


def _values(v, n, dev, message):
    t = torch.as_tensor(v, device=dev)
    if tuple(t.shape) != (n,):
        raise ValueError(message)
    t = t.to(torch.float64).contiguous()
    if n and not bool(torch.isfinite(t).all()):
        raise ValueError(message)
    return t


def triangulate(points, radii=None):
    """Delaunay tetrahedra [C,4] (int64, host) of ``points``; with ``radii``, only the
    cells whose six edges are no longer than the sum of their end points' radii
    (+1e-10) are kept (tetrahedra.py:19-31)."""
    from scipy.spatial import Delaunay

    points = np.asarray(points, np.float64)
    if len(points) < 4 or np.linalg.matrix_rank(points - points.mean(0)) < 3:
        raise ValueError("tetrahedral extraction needs >=4 noncoplanar points")
    cells = Delaunay(points).simplices.astype(np.int64)
    if radii is None:
        return cells
    r = np.asarray(radii)
    a, b = cells[:, EDGE_A], cells[:, EDGE_B]
    keep = (np.linalg.norm(points[a] - points[b], axis=-1) <= r[a] + r[b] + 1e-10).all(-1)
    return cells[keep]


def grid_points(means, quats, scales, opacities, *, seed_opacity_min=0.05, max_gaussians=None,
                tetra_extent=3.0):
    """The seed Gaussians (opacity >= ``seed_opacity_min``; the ``max_gaussians`` most
    opaque when there are more) and, on the device, their 9 grid points each (the
    centre, then the box corners in itertools.product((-1, 1), repeat=3) order) as
    float64 [n, 9, 3] with the float32 vertex radius max(scale) * extent [n]."""
    dev = _device_of(means)
    opacity = opacities.detach().reshape(-1).float().cpu().numpy()
    seeds = np.flatnonzero(opacity >= seed_opacity_min)
    if not len(seeds):
        raise ValueError("no Gaussian passes the mesh seed opacity threshold")
    if max_gaussians is not None and len(seeds) > max_gaussians:
        seeds = seeds[np.argsort(opacity[seeds])[-max_gaussians:]]
    with torch.cuda.device(dev), torch.no_grad():
        m, q, s = (t.detach().contiguous() for t in (means, quats, scales))
        ops._require_cuda_f32("mesh grid points", m, q, s)
        idx = torch.as_tensor(seeds.astype(np.int32), device=dev)
        n = len(seeds)
        pts = torch.empty((n, 9, 3), dtype=torch.float64, device=dev)
        radius = torch.empty((n,), dtype=torch.float64, device=dev)
        call("sf_b200_mesh_grid_points", _ptr(m), _ptr(q), _ptr(s), _ptr(idx), n, float(tetra_extent), _ptr(pts),
             _ptr(radius), _stream(dev))
    return pts, radius, n


def gaussian_grid(means, quats, scales, opacities, *, seed_opacity_min=0.05, max_gaussians=None,
                  tetra_extent=3.0):
    """(unique grid points [U,3] float64, tetrahedra [C,4] int64, seed count) as
    ``gaussian_grid`` (exporters.py:20-38) returns them, on the host."""
    pts, radius, n = grid_points(means, quats, scales, opacities, seed_opacity_min=seed_opacity_min,
                                 max_gaussians=max_gaussians, tetra_extent=tetra_extent)
    flat = pts.reshape(-1, 3).cpu().numpy()
    unique, inverse = np.unique(flat, axis=0, return_inverse=True)
    radii = np.zeros(len(unique))
    np.maximum.at(radii, inverse.reshape(-1), np.repeat(radius.cpu().numpy(), 9))
    return unique, triangulate(unique, radii), n


def marching_tetrahedra(points, cells, values, field, *, level=0.0, binary_steps=8, inside_greater=True):
    """Level set of a scalar field over tetrahedra, on the device.

    ``points`` [P,3] and ``values`` [P] (the field at the points) and ``cells`` [C,4] are
    tensors or arrays; ``field`` maps a CUDA float64 [M,3] tensor of bisection points to
    [M] finite values.  A point is inside when its value is >= ``level``
    (``inside_greater``) or <= ``level``.  Returns (vertices [U,3] float64, faces [F,3]
    int64) as CUDA tensors: one vertex per edge with one end inside, after
    ``binary_steps`` bisections, in ascending (low, high) vertex order; one face per cell
    with a 1/3 split and two per 2/2 split, in cell order, oriented away from the inside
    vertices, faces of area <= 1e-16 removed.  Invalid field values raise ``ValueError``
    (tetrahedra.py:34-109)."""
    dev = _device_of(points, cells, values)
    with torch.cuda.device(dev), torch.no_grad():
        stream = _stream(dev)
        pts = torch.as_tensor(points, device=dev).to(torch.float64).contiguous()
        cel = torch.as_tensor(cells, device=dev).to(torch.int32).reshape(-1, 4).contiguous()
        P, C = pts.shape[0], cel.shape[0]
        if pts.ndim != 2 or pts.shape[1] != 3:
            raise ValueError("points must be [P,3]")
        if C and (int(cel.min()) < 0 or int(cel.max()) >= P):
            raise ValueError("cells index outside the points")
        val = _values(values, P, dev, "field returned invalid vertex scalars")
        lvl, greater = float(level), int(bool(inside_greater))
        inside = torch.empty((P,), dtype=torch.uint8, device=dev)
        slot_off = torch.empty((C + 1,), dtype=torch.int64, device=dev)
        face_off = torch.empty((C + 1,), dtype=torch.int64, device=dev)
        ws = _workspace("sf_b200_mesh_count_workspace_bytes", C, dev)
        call("sf_b200_mesh_count", _ptr(val), P, _ptr(cel), C, lvl, greater, _ptr(inside), _ptr(slot_off),
             _ptr(face_off), _ptr(ws), ws.numel(), stream)
        n_slots, n_faces = (int(x) for x in torch.stack((slot_off[C], face_off[C])).cpu())
        if n_faces == 0:
            return (torch.empty((0, 3), dtype=torch.float64, device=dev),
                    torch.empty((0, 3), dtype=torch.int64, device=dev))

        edge_ids = torch.empty((n_slots,), dtype=torch.int32, device=dev)
        pairs = torch.empty((n_slots, 2), dtype=torch.int32, device=dev)
        low = torch.empty((n_slots, 3), dtype=torch.float64, device=dev)
        high = torch.empty((n_slots, 3), dtype=torch.float64, device=dev)
        low_in = torch.empty((n_slots,), dtype=torch.uint8, device=dev)
        count = torch.empty((1,), dtype=torch.int64, device=dev)
        ws = _workspace("sf_b200_mesh_edges_workspace_bytes", n_slots, dev)
        call("sf_b200_mesh_edges", _ptr(pts), P, _ptr(cel), C, _ptr(inside), _ptr(slot_off), n_slots,
             _ptr(edge_ids), _ptr(pairs), _ptr(low), _ptr(high), _ptr(low_in), _ptr(count), _ptr(ws), ws.numel(),
             stream)
        U = int(count.item())
        low, high, low_in = low[:U], high[:U], low_in[:U]
        mid = torch.empty((U, 3), dtype=torch.float64, device=dev)
        for _ in range(int(binary_steps)):
            call("sf_b200_mesh_midpoints", _ptr(low), _ptr(high), U, _ptr(mid), stream)
            v = _values(field(mid.clone()), U, dev, "field returned invalid bisection scalars")
            call("sf_b200_mesh_bisect", _ptr(low), _ptr(high), _ptr(low_in), U, _ptr(v), lvl, greater,
                 _stream(dev))

        vertices = torch.empty((U, 3), dtype=torch.float64, device=dev)
        faces = torch.empty((n_faces, 3), dtype=torch.int64, device=dev)
        ws = _workspace("sf_b200_mesh_faces_workspace_bytes", n_faces, dev)
        call("sf_b200_mesh_faces", _ptr(pts), _ptr(cel), C, _ptr(inside), _ptr(slot_off), _ptr(edge_ids), _ptr(low),
             _ptr(high), U, _ptr(face_off), n_faces, _ptr(vertices), _ptr(faces), _ptr(count), _ptr(ws),
             ws.numel(), stream)
        return vertices, faces[: int(count.item())]


def gof_mesh(means, quats, scales, opacities, origins, *, inverse_covariances=None, level=0.5, binary_steps=8,
             seed_opacity_min=0.05, max_gaussians=None, tetra_extent=3.0, culled=True):
    """The GOF exporter's extraction (exporters.py:41-88) on activated Gaussians
    (scales exponentiated, opacities after the sigmoid) and the training views' camera
    origins [V,3].  ``inverse_covariances`` defaults to inv(covariance(quats, scales)).
    The field is the culled opacity field through one ``ops.OpacityFieldPlan`` for the
    whole extraction (``culled``) or the brute-force one; the exporter's query and
    Gaussian chunking only bound the reference's memory and do not change the field, so
    every evaluation covers all queries at once.  Returns
    SimpleNamespace(vertices, faces, grid_vertices, tetrahedra, seeds)."""
    dev = _device_of(means)
    m, q, s, o, org = (t.detach().to(torch.float32).contiguous() for t in (means, quats, scales, opacities, origins))
    o = o.reshape(-1)
    if inverse_covariances is None:
        inverse_covariances = torch.linalg.inv(ops.covariance(q, s))
    inv = inverse_covariances.detach().to(torch.float32).contiguous()
    points, cells, seeds = gaussian_grid(m, q, s, o, seed_opacity_min=seed_opacity_min,
                                         max_gaussians=max_gaussians, tetra_extent=tetra_extent)
    if culled:
        plan = ops.OpacityFieldPlan(m, inv, o, org)

        def field_op(p, *args):
            return plan(p)
    else:
        field_op = ops.opacity_field

    def field(coordinates):
        # queries rounded to float32, as the reference's field converts them
        return field_op(coordinates.to(torch.float32).contiguous(), m, inv, o, org)

    pts = torch.as_tensor(points, device=dev)
    vertices, faces = marching_tetrahedra(pts, cells, field(pts), field, level=level, binary_steps=binary_steps,
                                          inside_greater=True)
    return SimpleNamespace(vertices=vertices, faces=faces, grid_vertices=len(points), tetrahedra=len(cells),
                           seeds=seeds)


def write_ply(path, vertices, faces):
    """Binary little-endian PLY: float32 x, y, z per vertex and a uchar-counted list of
    int32 indices per face, the layout ``write_mesh`` writes (src/splatforge/mesh/io.py:10-36)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    v = np.asarray(torch.as_tensor(vertices).cpu(), dtype="<f4")
    f = np.asarray(torch.as_tensor(faces).cpu(), dtype="<i4")
    if v.ndim != 2 or v.shape[1] != 3 or f.ndim != 2 or f.shape[1] != 3 or not np.isfinite(v).all():
        raise ValueError("mesh must contain finite Nx3 vertices and Mx3 faces")
    if len(f) and (f.min() < 0 or f.max() >= len(v)):
        raise ValueError("mesh indices are out of bounds")
    header = ("ply\nformat binary_little_endian 1.0\n"
              f"element vertex {len(v)}\nproperty float x\nproperty float y\nproperty float z\n"
              f"element face {len(f)}\nproperty list uchar int vertex_indices\nend_header\n")
    rec = np.empty(len(f), dtype=[("n", "u1"), ("idx", "<i4", (3,))])
    rec["n"] = 3
    rec["idx"] = f
    with path.open("wb") as out:
        out.write(header.encode("ascii"))
        out.write(v.tobytes())
        out.write(rec.tobytes())


class B200GOFExporter:
    """Drop-in for SplatForge's ``GOFExporter`` (exporters.py:41-102): the same
    ``export(pipeline, path, config)`` call, config fields (``level``,
    ``binary_steps``, ``seed_opacity_min``, ``max_gaussians``, ``tetra_extent``) and
    report, with the grid, the field and the marching stages on the device.
    ``culled_field=False`` selects the brute-force field."""

    def __init__(self, *, culled_field=True):
        self.culled_field = culled_field

    @torch.no_grad()
    def export(self, pipeline, path, config):
        model = pipeline.model
        inverse = torch.linalg.inv(pipeline.ops("gaussian.covariance@1", model.quats, model.scales))
        origins = torch.stack([pipeline.data.frames[i].camera.origin.to(model.device)
                               for i in pipeline.data.train_indices])
        mesh = gof_mesh(model.means, model.quats, model.scales, model.opacities, origins,
                        inverse_covariances=inverse, level=config.level, binary_steps=config.binary_steps,
                        seed_opacity_min=config.seed_opacity_min, max_gaussians=config.max_gaussians,
                        tetra_extent=config.tetra_extent, culled=self.culled_field)
        if not len(mesh.faces):
            raise ValueError("GOF level set is empty; training output is preserved")
        write_ply(path, mesh.vertices, mesh.faces)
        return {
            "exporter": "gof",
            "vertices": len(mesh.vertices),
            "faces": len(mesh.faces),
            "grid_vertices": mesh.grid_vertices,
            "tetrahedra": mesh.tetrahedra,
            "seed_gaussians": mesh.seeds,
            "level": config.level,
            "binary_steps": config.binary_steps,
            "training_views": len(origins),
            "path": str(path),
        }
