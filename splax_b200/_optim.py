"""Fused Adam for the training step around the render.

``Adam`` keeps optax.adam's state and update per parameter group (the reference's
scripts/train_colmap.py:639-645 builds one optax.adam per group: means, scales, quats, colors,
opacities, each with its own learning rate) and applies every group in one library launch
(``splax_adam_step``). There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import torch

from splax_b200 import _lib


class Adam:
    """In-place Adam over CUDA fp32 parameters with one learning rate per tensor.

    Matches ``optax.adam(lr, b1, b2, eps)`` (eps_root 0): moments start at zero and the bias
    correction uses the update count. ``step(grads)`` takes the gradients explicitly or reads
    each parameter's ``.grad``.
    """

    def __init__(self, params: Sequence[torch.Tensor], lrs: Sequence[float] | float,
                 b1: float = 0.9, b2: float = 0.999, eps: float = 1e-8):
        self.params = list(params)
        if isinstance(lrs, (int, float)):
            lrs = [float(lrs)] * len(self.params)
        if len(lrs) != len(self.params):
            raise ValueError(f"{len(lrs)} learning rates for {len(self.params)} parameters")
        for p in self.params:
            _lib.require_cuda(p)
            if p.dtype != torch.float32 or not p.is_contiguous():
                raise ValueError("Adam needs contiguous fp32 parameters")
        self.lrs = [float(x) for x in lrs]
        self.b1, self.b2, self.eps = float(b1), float(b2), float(eps)
        self.exp_avg = [torch.zeros_like(p) for p in self.params]
        self.exp_avg_sq = [torch.zeros_like(p) for p in self.params]
        self.count = 0

    @torch.no_grad()
    def step(self, grads: Sequence[torch.Tensor] | None = None) -> None:
        if grads is None:
            grads = [p.grad for p in self.params]
        gs = []
        for p, g in zip(self.params, grads):
            if g is None:
                raise ValueError("a parameter has no gradient")
            if g.shape != p.shape:
                raise ValueError(f"gradient {tuple(g.shape)} for parameter {tuple(p.shape)}")
            gs.append(g.detach().to(torch.float32).contiguous())
        self.count += 1
        k = len(self.params)
        ptrs = lambda ts: (ctypes.c_void_p * k)(*[t.data_ptr() for t in ts])  # noqa: E731
        sizes = (ctypes.c_int64 * k)(*[p.numel() for p in self.params])
        lrs = (ctypes.c_float * k)(*self.lrs)
        lib = _lib.load()
        dev = self.params[0].device
        with torch.cuda.device(dev):
            rc = lib.splax_adam_step(k, ptrs(self.params), ptrs(gs), ptrs(self.exp_avg),
                                     ptrs(self.exp_avg_sq), sizes, lrs, self.count, self.b1,
                                     self.b2, self.eps, _lib.stream_of(self.params[0]))
        _lib.check(rc)
