"""Fused image losses for training steps around the render.

``mse_loss`` is the mean-squared-error objective of the benchmark configurations 1 and 2,
sum((img - target)^2) / denom, as one library kernel per direction (no counterpart in the
reference, whose callers take the loss in JAX). Differentiable with respect to ``img``; the
target gets no gradient.
"""

from __future__ import annotations

import torch

from splax_b200 import _lib


class _MSELossFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img, target, denom):
        dev = _lib.require_cuda(img, target)
        if img.shape != target.shape:
            raise ValueError(f"img {tuple(img.shape)} and target {tuple(target.shape)} differ")
        a = img.detach().to(torch.float32).contiguous()
        t = target.detach().to(torch.float32).contiguous()
        loss = torch.empty((), device=dev, dtype=torch.float32)
        lib = _lib.load()
        with torch.cuda.device(dev):
            rc = lib.splax_mse_loss(_lib.ptr(a), _lib.ptr(t), a.numel(), float(denom),
                                    _lib.ptr(loss), _lib.stream_of(a))
        _lib.check(rc)
        ctx.save_for_backward(a, t)
        ctx.denom = float(denom)
        ctx.img_dtype = img.dtype
        return loss

    @staticmethod
    def backward(ctx, v_loss):
        a, t = ctx.saved_tensors
        g = torch.empty_like(a)
        v = v_loss.detach().to(torch.float32).reshape(()).contiguous()
        lib = _lib.load()
        with torch.cuda.device(a.device):
            rc = lib.splax_mse_loss_bwd(_lib.ptr(a), _lib.ptr(t), a.numel(), ctx.denom,
                                        _lib.ptr(v), _lib.ptr(g), _lib.stream_of(a))
        _lib.check(rc)
        return g.to(ctx.img_dtype), None, None


def mse_loss(img: torch.Tensor, target: torch.Tensor, *, denom: float | None = None) -> torch.Tensor:
    """sum((img - target)^2) / denom as a 0-d tensor (denom defaults to img.numel(), the
    mean). Pass the global element count as ``denom`` when each rank holds a camera shard."""
    d = float(img.numel() if denom is None else denom)
    if not d > 0:
        raise ValueError(f"denom must be positive, got {d}")
    return _MSELossFn.apply(img, target, d)
