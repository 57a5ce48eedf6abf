"""The oracle renderer run tile batch by tile batch on any device (test infrastructure).

``oracle.render.render`` builds one autograd graph over the whole frame, which is fine
for crops on the CPU but holds every tile batch's intermediates at once.  For whole
1080p frames of the million-Gaussian scene this helper evaluates the same
projection, the same padded tile batches and the same per-batch equations
(``oracle.render.prepare`` / ``tile_batches`` / ``render_batch``), but back-propagates
each batch as soon as it is built, into detached copies of the projected per-Gaussian
tensors, and then runs the projection's backward once.  This is the checkpointing the
reference's own ``BatchedTorchRenderer`` applies per tile batch
(src/splatforge/studio/batched_renderer.py:380-395): the images and gradients are the
ones the whole-frame graph gives, summed in a different order.
"""

from __future__ import annotations

import torch

from oracle import render as oracle_render
from splatforge_b200 import scenes
from tests._util import CHANNELS, PARAM_NAMES

# the per-Gaussian tensors ``render_batch`` gathers by tile list
PROJECTED = ("xy", "conic", "colors", "ray_colors", "opacity", "m", "normals", "gain", "qinv", "plane")


def _device_view(params, device, activation_device):
    """Raw-parameter leaves on ``activation_device``, activated there, then a
    differentiable copy to ``device``.  A kernel run that activates on the same device
    sees bit-identical inputs (torch's CUDA and CPU ``exp`` can differ in the last bit)."""
    p = params.detach_clone().to(activation_device).requires_grad_()
    v = scenes.activated(p)
    view = scenes.View(*(t.to(device) for t in (v.means, v.quats, v.scales, v.opacities, v.sh)), params.sh_degree)
    return p, view


def render(params, cam, mode, distortions, sel, ups, *, device, settings=None, trunc_sigma=2.0,
           activation_device="cpu"):
    """Oracle images (dict of HWC tensors on ``device``) and gradients of
    ``sum_ch <image_ch, ups_ch>`` with respect to the raw parameters (tensors on
    ``activation_device``, keyed by PARAM_NAMES) plus ``means2d_grad`` and ``absgrad``
    (CPU tensors)."""
    p, view = _device_view(params, device, activation_device)
    camd = cam.to(device)
    ctx = oracle_render.prepare(view, camd, mode=mode, settings=settings,
                                selected=None if sel is None else sel.to(device),
                                distortions=distortions, trunc_sigma=trunc_sigma)
    graph = {k: ctx[k] for k in PROJECTED if ctx[k].requires_grad}
    for k, t in graph.items():
        leaf = t.detach().requires_grad_()
        if k == "xy":
            leaf.absgrad = torch.zeros_like(leaf)
        ctx[k] = leaf
    H, W = cam.height, cam.width
    ts = ctx["settings"].tile_size
    cols = (W + ts - 1) // ts
    upstream = torch.cat([ups[ch].to(device) for ch in CHANNELS], -1)  # [H, W, 13]
    image = torch.empty_like(upstream)
    for tiles, longest in oracle_render.tile_batches(ctx):
        blocks = []
        for t in tiles:
            top, left = (t // cols) * ts, (t % cols) * ts
            h, w = min(ts, H - top), min(ts, W - left)
            blocks.append((top, left, h, w))
        out = oracle_render.render_batch(ctx, tiles, longest)
        up = torch.stack([upstream[a:a + h, b:b + w].reshape(h * w, -1) for a, b, h, w in blocks])
        if out.requires_grad:
            (out * up).sum().backward()
        out = out.detach()
        for row, (a, b, h, w) in enumerate(blocks):
            image[a:a + h, b:b + w] = out[row].reshape(h, w, -1)
    leaves = {k: ctx[k] for k in graph}
    pairs = [(graph[k], leaves[k].grad) for k in graph if leaves[k].grad is not None]
    torch.autograd.backward([a for a, _ in pairs], [g for _, g in pairs])
    parts = torch.split(image, [3 if ch in ("rgb", "normals") else 1 for ch in CHANNELS], -1)
    images = dict(zip(CHANNELS, parts))
    grads = {name: t.grad for name, t in zip(PARAM_NAMES, p.tensors())}
    xy = leaves.get("xy")
    grads["means2d_grad"] = xy.grad.cpu() if xy is not None and xy.grad is not None else None
    grads["absgrad"] = xy.absgrad.cpu() if xy is not None else None
    return images, grads, ctx
