"""Fused image losses for training steps around the render.

``mse_loss`` is the mean-squared-error objective of the benchmark configurations 1 and 2,
sum((img - target)^2) / denom; ``l1_dssim_loss`` is the photometric loss of the batched
training step (config 3; scripts/train_colmap.py:202-221), (1 - lambda) L1 + lambda D-SSIM.
Each is one library kernel per direction (no counterpart in the reference, whose callers take
the loss in JAX). Differentiable with respect to the image; the target gets no gradient.
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


class _L1DssimFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img, target, views_total, ssim_lambda):
        dev = _lib.require_cuda(img, target)
        if img.shape != target.shape or img.dim() not in (3, 4) or img.shape[-1] != 3:
            raise ValueError(f"img {tuple(img.shape)} and target {tuple(target.shape)} must be "
                             "equal (H, W, 3) or (B, H, W, 3)")
        a = img.detach().to(torch.float32).contiguous()
        t = target.detach().to(torch.float32).contiguous()
        B = a.shape[0] if a.dim() == 4 else 1
        H, W = a.shape[-3], a.shape[-2]
        loss = torch.empty((), device=dev, dtype=torch.float32)
        lib = _lib.load()
        # a training step takes the gradient next: compute it with the loss in one pass (for a
        # unit cotangent; backward scales it)
        fused = bool(ctx.needs_input_grad[0])
        with torch.cuda.device(dev):
            if fused:
                g = torch.empty_like(a)
                rc = lib.splax_l1_dssim_loss_and_grad(
                    _lib.ptr(a), _lib.ptr(t), B, H, W, int(views_total), float(ssim_lambda),
                    _lib.ptr(loss), _lib.ptr(g), _lib.stream_of(a))
            else:
                rc = lib.splax_l1_dssim_loss(_lib.ptr(a), _lib.ptr(t), B, H, W, int(views_total),
                                             float(ssim_lambda), _lib.ptr(loss),
                                             _lib.stream_of(a))
        _lib.check(rc)
        if fused:
            ctx.save_for_backward(g)
        else:
            ctx.save_for_backward(a, t)
        ctx.fused = fused
        ctx.args = (B, H, W, int(views_total), float(ssim_lambda), img.dtype)
        return loss

    @staticmethod
    def backward(ctx, v_loss):
        B, H, W, views_total, lam, dtype = ctx.args
        v = v_loss.detach().to(torch.float32).reshape(()).contiguous()
        if ctx.fused:
            (g,) = ctx.saved_tensors
            return (g * v).to(dtype), None, None, None  # out of place: backward may run twice
        a, t = ctx.saved_tensors
        g = torch.empty_like(a)
        lib = _lib.load()
        with torch.cuda.device(a.device):
            rc = lib.splax_l1_dssim_loss_bwd(_lib.ptr(a), _lib.ptr(t), B, H, W, views_total, lam,
                                             _lib.ptr(v), _lib.ptr(g), _lib.stream_of(a))
        _lib.check(rc)
        return g.to(dtype), None, None, None


def l1_dssim_loss(img: torch.Tensor, target: torch.Tensor, *, ssim_lambda: float = 0.2,
                  views_total: int | None = None) -> torch.Tensor:
    """(1 - ssim_lambda) mean|img - target| + ssim_lambda (1 - SSIM), averaged over the views of
    a (B, H, W, 3) stack (or one (H, W, 3) view), as the reference's make_step computes it with
    dm_pix.ssim. With camera shards pass the global view count as ``views_total``: each rank
    then gets its additive share of the loss and the global gradient of its images."""
    B = img.shape[0] if img.dim() == 4 else 1
    V = B if views_total is None else int(views_total)
    if V < B:
        raise ValueError(f"views_total={V} is less than the {B} views given")
    return _L1DssimFn.apply(img, target, V, float(ssim_lambda))
