"""Shared helpers for the parity tests."""

from __future__ import annotations

import numpy as np
import torch

from splatforge_b200 import scenes

CHANNELS = ("rgb", "alpha", "depth", "normals", "distortion_l1", "distortion_l2",
            "median_depth", "ray_color", "ambiguity_mask")
PARAM_NAMES = ("means", "log_scales", "quats", "opacity_logits", "sh")


def params_from(fix, prefix="params/"):
    t = [torch.from_numpy(fix[prefix + n]) for n in PARAM_NAMES]
    return scenes.SceneParams(*t, sh_degree=3)


def camera_from(fix, prefix):
    w, h = (int(v) for v in fix[prefix + "size"])
    return scenes.PinholeCamera(
        torch.from_numpy(fix[prefix + "K"]), torch.from_numpy(fix[prefix + "w2c"]), w, h
    )


def linear_loss(outputs, ups):
    """sum over channels of <image, upstream> (the fixtures' seeded loss)."""
    loss = 0
    for ch in CHANNELS:
        loss = loss + (outputs[ch] * ups[ch].to(outputs[ch].device)).sum()
    return loss


def rel_err(a, b, eps=1e-12):
    a = torch.as_tensor(a, dtype=torch.float64)
    b = torch.as_tensor(b, dtype=torch.float64)
    return float((a - b).norm() / max(float(b.norm()), eps))


def median_mismatch_ok(got, want, tol, frac=0.002):
    """Median depth is discontinuous where the cumulative weight sits at 0.5;
    allow a tiny fraction of pixels to pick the neighbouring sample."""
    bad = (torch.as_tensor(got) - torch.as_tensor(want)).abs() > tol
    return float(bad.float().mean()) <= frac


def numpy(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def reference_source():
    """A directory from which the reference package ``splatforge`` imports, or None:
    the ``SPLATFORGE_SRC`` environment variable (the reference's ``src`` directory), else
    the copy ``pip install --target baseline/_ref`` puts beside this repository."""
    import os
    from pathlib import Path

    env = os.environ.get("SPLATFORGE_SRC")
    candidates = [Path(env)] if env else []
    candidates.append(Path(__file__).resolve().parent.parent / "baseline" / "_ref")
    for c in candidates:
        if (c / "splatforge").is_dir():
            return c
    return None
