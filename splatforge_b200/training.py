"""The training-step operations on either side of the renderer, on the device.

* ``observe(densifier, output, model)`` -- ``GaussianDensifier.observe``
  (src/splatforge/studio/densification.py:18-43): the norm of each Gaussian's
  projected-mean gradient (``.absgrad`` or ``.grad`` per ``config.absolute_gradients``,
  scaled to NDC units when ``config.gradient_space == "ndc"``) is added to
  ``densifier.gradient`` where its projected radius is positive, and
  ``densifier.observations`` counts those views; one kernel, in place.
* ``normal_consistency(output, camera, ops, mask)`` -- the normal-consistency loss
  (src/splatforge/studio/losses.py:45-53): normals from the rendered depth
  (geometry.depth_normals@1), kept where they are valid, alpha > 0.1 and mask > 0, against
  the rendered normal numerator (alpha - n_num . n_depth) or the unit normals
  (1 - n . n_depth); the masked mean (losses.py:9-12).  Differentiable in depth, alpha and
  the normals; one forward and one backward pass over the pixels plus the depth-normal
  adjoint.
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import call
from .ops import _require_cuda_f32
from .rasterizer import _ptr, _stream


def observe(densifier, output, model):
    """In-place densification statistics with the reference's semantics and errors."""
    projected = output.projected_means
    if projected is None:
        return
    config = densifier.config
    gradient = getattr(projected, "absgrad", None) if config.absolute_gradients else projected.grad
    if gradient is None:
        return
    gradient = gradient.detach().reshape(-1, 2)
    if len(gradient) != model.count:
        raise ValueError("renderer densification statistics do not match Gaussian count")
    radii = output.projected_radii.detach().reshape(-1).to(torch.float32).contiguous()
    g = gradient.to(torch.float32).contiguous()
    acc, obs = densifier.gradient, densifier.observations
    _require_cuda_f32("densify observe", g, radii, acc, obs)
    if not (acc.is_contiguous() and obs.is_contiguous()):
        raise ValueError("densify observe: accumulators must be contiguous")
    sx, sy = (output.rgb.shape[1] / 2, output.rgb.shape[0] / 2) if config.gradient_space == "ndc" else (1.0, 1.0)
    dev = g.device
    with torch.cuda.device(dev):
        call("sf_b200_densify_observe", _ptr(g), _ptr(radii), g.shape[0], ctypes.c_float(sx), ctypes.c_float(sy),
             _ptr(acc), _ptr(obs), _stream(dev))


class _NormalConsistency(torch.autograd.Function):
    @staticmethod
    def forward(ctx, depth, K, alpha, vector, mask, numerator):
        H, W = depth.shape
        dev = depth.device
        size = ctypes.c_size_t()
        call("sf_b200_normal_consistency_workspace_bytes", W, H, ctypes.byref(size))
        ws = torch.empty((max(size.value, 1),), device=dev, dtype=torch.uint8)
        loss = torch.empty((), device=dev, dtype=torch.float32)
        count = torch.empty((), device=dev, dtype=torch.int64)
        num, unit = (vector, None) if numerator else (None, vector)
        with torch.cuda.device(dev):
            call("sf_b200_normal_consistency", _ptr(depth), _ptr(K), W, H, _ptr(alpha), _ptr(num), _ptr(unit),
                 _ptr(mask), _ptr(loss), _ptr(count), _ptr(ws), ws.numel(), _stream(dev))
        ctx.save_for_backward(depth, K, alpha, vector, mask, count)
        ctx.ws, ctx.numerator = ws, numerator
        return loss

    @staticmethod
    def backward(ctx, g_loss):
        depth, K, alpha, vector, mask, count = ctx.saved_tensors
        H, W = depth.shape
        dev = depth.device
        g = g_loss.to(torch.float32).contiguous()
        g_depth = torch.empty_like(depth)
        g_alpha = torch.empty_like(alpha) if ctx.numerator else None
        g_vec = torch.empty_like(vector)
        g_normals = torch.empty_like(vector)
        num, unit = (vector, None) if ctx.numerator else (None, vector)
        with torch.cuda.device(dev):
            call("sf_b200_normal_consistency_backward", _ptr(depth), _ptr(K), W, H, _ptr(alpha), _ptr(num),
                 _ptr(unit), _ptr(mask), _ptr(g), _ptr(count), _ptr(g_depth), _ptr(g_alpha), _ptr(g_vec),
                 _ptr(g_normals), _ptr(ctx.ws), ctx.ws.numel(), _stream(dev))
        return g_depth, None, g_alpha, g_vec, None, None


def normal_consistency(output, camera, ops=None, mask=None):
    """Scalar loss of losses.py:45-53 on a ``RenderOutput`` (depth, alpha, normals [H,W,*],
    ``normal_numerator`` or None) and its camera (``K``); ``mask`` [H,W,1] or [H,W].
    ``ops`` is accepted for the reference's signature; the depth normals come from this
    library's kernel."""
    del ops
    depth = output.depth.squeeze(-1)
    alpha = output.alpha.squeeze(-1)
    numer = getattr(output, "normal_numerator", None)
    vector = numer if numer is not None else output.normals
    m = mask.squeeze(-1) if mask is not None else torch.ones_like(depth)
    K = camera.K.to(device=depth.device, dtype=torch.float32)
    _require_cuda_f32("normal consistency", depth, alpha, vector, m.to(torch.float32), K)
    args = [t.contiguous() for t in (depth, K, alpha, vector, m.to(torch.float32))]
    return _NormalConsistency.apply(*args, numer is not None)
