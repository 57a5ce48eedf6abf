"""Seeded synthetic Gaussian scenes and pinhole cameras.

The shapes and value distributions follow the five workloads this provider is
measured on (no public dataset is used; every tensor is generated from a seed):

* ``demo48``   48 Gaussians, means U[-1,1]^3, log-scales N(-2.5, 0.3), opacity 0.7,
               eight 24x24 views at 60 deg on a radius-3 sphere.
* ``surfaces`` Gaussians sampled on 10 random spheres and 10 random square planes
               with N(0, 0.01) jitter, log-scales N(-4, 0.5), opacity sigmoid(N(0, 1.5)).

All scenes carry SH degree 3 with DC coefficients N(0.5, 0.1) and higher bands
N(0, 0.05).  Cameras use the OpenCV convention of the reference
(``src/splatforge/gaussian/semantics.json:5``: x right, y down, z forward,
world-to-camera matrices) and ``K = [[f,0,W/2],[0,f,H/2],[0,0,1]]`` with
``f = (W/2) / tan(fov/2)`` (horizontal field of view).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class SceneParams:
    """Raw trainable parameters, named as in ``GaussianScene`` (studio/model.py:44-57)."""

    means: torch.Tensor
    log_scales: torch.Tensor
    quats: torch.Tensor
    opacity_logits: torch.Tensor
    sh: torch.Tensor
    sh_degree: int = 3

    def tensors(self):
        return (self.means, self.log_scales, self.quats, self.opacity_logits, self.sh)

    def to(self, device):
        return SceneParams(
            *(t.to(device) for t in self.tensors()), sh_degree=self.sh_degree
        )

    def requires_grad_(self, flag=True):
        for t in self.tensors():
            t.requires_grad_(flag)
        return self

    def detach_clone(self):
        return SceneParams(
            *(t.detach().clone() for t in self.tensors()), sh_degree=self.sh_degree
        )


@dataclass
class View:
    """Activated Gaussian attributes, field-for-field ``GaussianView`` (studio/renderers.py:20-27)."""

    means: torch.Tensor
    quats: torch.Tensor
    scales: torch.Tensor
    opacities: torch.Tensor
    sh: torch.Tensor
    sh_degree: int


def activated(params: SceneParams) -> View:
    """``scales = exp(log_scales)``, ``opacities = sigmoid(logits)`` (studio/model.py:73-79)."""
    return View(
        params.means,
        params.quats,
        params.log_scales.exp(),
        params.opacity_logits.sigmoid(),
        params.sh,
        params.sh_degree,
    )


@dataclass(frozen=True)
class PinholeCamera:
    """Field-for-field ``Camera`` (studio/cameras.py:8-22)."""

    K: torch.Tensor
    world_to_camera: torch.Tensor
    width: int
    height: int
    name: str = ""

    @property
    def camera_to_world(self):
        return torch.linalg.inv(self.world_to_camera)

    @property
    def origin(self):
        return self.camera_to_world[:3, 3]

    def to(self, device, dtype=torch.float32):
        return PinholeCamera(
            self.K.to(device=device, dtype=dtype),
            self.world_to_camera.to(device=device, dtype=dtype),
            self.width,
            self.height,
            self.name,
        )

    def crop(self, left: int, top: int, width: int, height: int):
        """A sub-window camera: same rays for the covered pixels (principal point shift)."""
        K = self.K.clone()
        K[0, 2] -= left
        K[1, 2] -= top
        return PinholeCamera(K, self.world_to_camera.clone(), width, height, self.name)


def _sh(rng, n, degree):
    coeffs = (degree + 1) ** 2
    sh = rng.normal(0.0, 0.05, size=(n, coeffs, 3))
    sh[:, 0, :] = rng.normal(0.5, 0.1, size=(n, 3))
    return sh


def _quats(rng, n):
    q = rng.normal(size=(n, 4))
    return q / np.linalg.norm(q, axis=-1, keepdims=True)


def demo48(seed: int = 0, n: int = 48) -> SceneParams:
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1.0, 1.0, size=(n, 3))
    log_scales = rng.normal(-2.5, 0.3, size=(n, 3))
    quats = _quats(rng, n)
    opacity = np.full(n, 0.7)
    logits = np.log(opacity / (1 - opacity))
    sh = _sh(rng, n, 3)
    return _pack(means, log_scales, quats, logits, sh)


def surface_primitives(seed: int, count: int = 20):
    """10 spheres (centre U[-1,1]^3, radius U[0.1,0.5]) and 10 square planes
    (centre U[-1,1]^3, random normal, side U[0.5,1.5])."""
    rng = np.random.default_rng(seed + 7919)
    prims = []
    for k in range(count):
        centre = rng.uniform(-1.0, 1.0, size=3)
        if k < count // 2:
            radius = rng.uniform(0.1, 0.5)
            prims.append(("sphere", centre, radius, 4 * math.pi * radius * radius))
        else:
            normal = rng.normal(size=3)
            normal /= np.linalg.norm(normal)
            side = rng.uniform(0.5, 1.5)
            prims.append(("plane", centre, (normal, side), side * side))
    return prims


def surfaces(n: int, seed: int = 0) -> SceneParams:
    rng = np.random.default_rng(seed)
    prims = surface_primitives(seed)
    areas = np.array([p[3] for p in prims])
    counts = np.floor(n * areas / areas.sum()).astype(np.int64)
    counts[np.argmax(areas)] += n - counts.sum()
    pts = []
    for (kind, centre, shape, _), m in zip(prims, counts):
        if m == 0:
            continue
        if kind == "sphere":
            d = rng.normal(size=(m, 3))
            d /= np.linalg.norm(d, axis=-1, keepdims=True)
            pts.append(centre + shape * d)
        else:
            normal, side = shape
            helper = np.array([1.0, 0.0, 0.0]) if abs(normal[0]) < 0.9 else np.array([0.0, 1.0, 0.0])
            u = np.cross(normal, helper)
            u /= np.linalg.norm(u)
            v = np.cross(normal, u)
            a = rng.uniform(-0.5, 0.5, size=(m, 1)) * side
            b = rng.uniform(-0.5, 0.5, size=(m, 1)) * side
            pts.append(centre + a * u + b * v)
    means = np.concatenate(pts, 0)
    means = means[rng.permutation(len(means))]
    means = means + rng.normal(0.0, 0.01, size=means.shape)
    log_scales = rng.normal(-4.0, 0.5, size=(n, 3))
    quats = _quats(rng, n)
    logits = rng.normal(0.0, 1.5, size=n)
    sh = _sh(rng, n, 3)
    return _pack(means, log_scales, quats, logits, sh)


def _pack(means, log_scales, quats, logits, sh) -> SceneParams:
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return SceneParams(f(means), f(log_scales), f(quats), f(logits), f(sh), 3)


def look_at(position, target=(0.0, 0.0, 0.0)):
    """OpenCV world-to-camera: rows (right, down, forward); t = -R p."""
    position = np.asarray(position, dtype=np.float64)
    forward = np.asarray(target, dtype=np.float64) - position
    forward /= np.linalg.norm(forward)
    up = np.array([0.0, 0.0, 1.0])
    if abs(forward @ up) > 0.99:
        up = np.array([0.0, 1.0, 0.0])
    right = np.cross(forward, up)
    right /= np.linalg.norm(right)
    down = np.cross(forward, right)
    R = np.stack((right, down, forward), 0)
    w2c = np.eye(4)
    w2c[:3, :3] = R
    w2c[:3, 3] = -R @ position
    return w2c


def intrinsics(width, height, fov_deg):
    f = (width / 2.0) / math.tan(math.radians(fov_deg) / 2.0)
    return np.array([[f, 0.0, width / 2.0], [0.0, f, height / 2.0], [0.0, 0.0, 1.0]])


def orbit_cameras(count, width, height, fov_deg, *, radius=3.0, seed=0, radius_range=None):
    rng = np.random.default_rng(seed + 104729)
    cams = []
    for k in range(count):
        d = rng.normal(size=3)
        d /= np.linalg.norm(d)
        r = radius if radius_range is None else rng.uniform(*radius_range)
        w2c = look_at(d * r)
        K = intrinsics(width, height, fov_deg)
        cams.append(
            PinholeCamera(
                torch.tensor(K, dtype=torch.float32),
                torch.tensor(w2c, dtype=torch.float32),
                width,
                height,
                f"view{k:03d}",
            )
        )
    return cams


# --- named workloads --------------------------------------------------------

def rotations(quats: torch.Tensor) -> torch.Tensor:
    """[N,4] wxyz (normalised here) -> [N,3,3] rotation matrices."""
    q = quats / quats.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    w, x, y, z = q.unbind(-1)
    return torch.stack(
        (
            1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
            2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
            2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
        ),
        -1,
    ).reshape(-1, 3, 3)


def inverse_covariances(params: SceneParams) -> torch.Tensor:
    """[N,3,3] inverse covariances R diag(1/s^2) R^T of the activated scales."""
    R = rotations(params.quats)
    inv_s2 = torch.exp(-2.0 * params.log_scales)
    return (R * inv_s2[:, None, :]) @ R.transpose(-1, -2)


def field_queries(params: SceneParams, n_uniform: int, *, extent: float = 3.0, seed: int = 0) -> torch.Tensor:
    """Query points of a GOF extraction grid: every Gaussian's centre and the 8 corners
    of its extent-sigma box along its own axes (the shape of the exporter's
    gaussian_grid, src/splatforge/studio/exporters.py:20-38, without deduplication),
    plus ``n_uniform`` points uniform in the bounding box of the means."""
    R = rotations(params.quats)
    s = torch.exp(params.log_scales)
    signs = torch.tensor([[0.0, 0.0, 0.0]] + [[a, b, c] for a in (-1.0, 1.0) for b in (-1.0, 1.0) for c in (-1.0, 1.0)])
    local = signs[None] * s[:, None, :] * extent                      # [N, 9, 3]
    pts = params.means[:, None, :] + torch.einsum("nij,nkj->nki", R, local)
    g = torch.Generator().manual_seed(seed + 2718)
    lo, hi = params.means.min(0).values, params.means.max(0).values
    uni = lo + (hi - lo) * torch.rand(n_uniform, 3, generator=g)
    return torch.cat((pts.reshape(-1, 3), uni), 0).contiguous()


def workload(name: str, seed: int = 0):
    """Returns ``(SceneParams, [PinholeCamera])`` for a named workload."""
    if name == "demo48":
        return demo48(seed), orbit_cameras(8, 24, 24, 60.0, radius=3.0, seed=seed)
    if name == "surfaces100k_800":
        return surfaces(100_000, seed), orbit_cameras(1, 800, 800, 50.0, radius=3.0, seed=seed)
    if name == "surfaces1m_1080p":
        return surfaces(1_000_000, seed), orbit_cameras(1, 1920, 1080, 60.0, radius=3.0, seed=seed)
    if name == "surfaces3m_views64":
        return surfaces(3_000_000, seed), orbit_cameras(
            64, 1600, 1064, 60.0, seed=seed, radius_range=(2.5, 4.0)
        )
    if name == "mesh100k_views32":
        # the GOF mesh-extraction workload: 100k Gaussians, 32 training-view origins
        return surfaces(100_000, seed), orbit_cameras(32, 1280, 720, 60.0, radius=3.0, seed=seed)
    if name == "field2m_views32":
        # the GOF opacity-field workload: 2M Gaussians, 32 training-view origins
        return surfaces(2_000_000, seed), orbit_cameras(32, 1280, 720, 60.0, radius=3.0, seed=seed)
    raise ValueError(f"unknown workload {name}")
