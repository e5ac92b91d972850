"""CPU restatement of the config-3 photometric loss, for tests only (never used by the product
path): (1 - lambda) L1 + lambda D-SSIM as the reference's make_step takes it
(scripts/train_colmap.py:202-221), with SSIM per its published definition (Wang et al. 2004)
in the form of the reference's dependency dm_pix 0.4.5 (pixi.lock; absent here, so its own
outputs cannot be run): an 11-tap Gaussian window of sigma 1.5 applied separably with VALID
extent, variances floored at eps_f32^2, the covariance clamped in magnitude to
sqrt(var_a var_b), k1 = 0.01, k2 = 0.03, max_val = 1, and the map averaged over positions and
channels. Evaluated in float64 on the CPU with torch; the gradient is torch autograd of this
forward (an independent derivation from the CUDA kernel's hand-written adjoint).

Parity unpinned: with dm_pix missing, the restatement is checked against known answers only
(identical images, constant images in closed form, the window's moments).
"""

from __future__ import annotations

import math

import numpy as np
import torch

EPS2 = float(np.finfo(np.float32).eps) ** 2
C1 = 0.01 ** 2
C2 = 0.03 ** 2


def window(size: int = 11, sigma: float = 1.5) -> np.ndarray:
    hw = size // 2
    f = np.exp(-0.5 * ((np.arange(size) - hw) / sigma) ** 2)
    return f / f.sum()


def _blur(z: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """VALID separable window over (H, W) of a (C, H, W) tensor."""
    k = w.numel()
    zh = z.unfold(2, k, 1) @ w          # along W: (C, H, W-k+1)
    return (zh.unfold(1, k, 1) @ w)     # along H: (C, H-k+1, W-k+1)


def ssim_map(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """SSIM map of (H, W, 3) images, (3, H-10, W-10)."""
    w = torch.tensor(window(), dtype=a.dtype)
    A, Bm = a.permute(2, 0, 1), b.permute(2, 0, 1)
    mu0, mu1 = _blur(A, w), _blur(Bm, w)
    mu00, mu11, mu01 = mu0 * mu0, mu1 * mu1, mu0 * mu1
    s00 = torch.clamp_min(_blur(A * A, w) - mu00, EPS2)
    s11 = torch.clamp_min(_blur(Bm * Bm, w) - mu11, EPS2)
    r01 = _blur(A * Bm, w) - mu01
    s01 = torch.sign(r01) * torch.minimum(torch.sqrt(s00 * s11), torch.abs(r01))
    return ((2 * mu01 + C1) * (2 * s01 + C2)) / ((mu00 + mu11 + C1) * (s00 + s11 + C2))


def l1_dssim(img: np.ndarray, target: np.ndarray, ssim_lambda: float = 0.2,
             views_total: int | None = None) -> tuple[float, np.ndarray]:
    """Loss share and its gradient w.r.t. img for a (B, H, W, 3) stack, float64."""
    a = torch.tensor(np.asarray(img, np.float64), requires_grad=True)
    t = torch.tensor(np.asarray(target, np.float64))
    B = a.shape[0]
    V = B if views_total is None else views_total
    l1 = sum(torch.abs(a[i] - t[i]).mean() for i in range(B)) / V
    dssim = sum(1.0 - ssim_map(a[i], t[i]).mean() for i in range(B)) / V
    loss = (1.0 - ssim_lambda) * l1 + ssim_lambda * dssim
    loss.backward()
    return float(loss.detach()), a.grad.numpy()


def constant_ssim(ca: float, cb: float) -> float:
    """Closed form of SSIM for two constant images: zero variances floored at eps^2, zero
    covariance."""
    return ((2 * ca * cb + C1) * C2) / ((ca * ca + cb * cb + C1) * (2 * EPS2 + C2))


def adam(param, grad, m, v, step: int, lr: float, b1: float = 0.9, b2: float = 0.999,
         eps: float = 1e-8):
    """optax.adam's update (optax 0.2.8, scale_by_adam + scale(-lr)) in float64: moments
    m = b1 m + (1 - b1) g, v = b2 v + (1 - b2) g^2, bias-corrected by 1 - b^step,
    update = -lr m_hat / (sqrt(v_hat) + eps). Returns (param', m', v').

    The decay constants are the fp32 values an fp32 optax state uses: b1, b2 rounded to fp32
    and 1 - b formed in fp32 (1 - 0.999f is 9.9998713e-4, not 1e-3)."""
    f32 = np.float32
    b1f, b2f = f32(b1), f32(b2)
    c1, c2 = float(f32(1) - b1f), float(f32(1) - b2f)
    g = np.asarray(grad, np.float64)
    m2 = float(b1f) * np.asarray(m, np.float64) + c1 * g
    v2 = float(b2f) * np.asarray(v, np.float64) + c2 * g * g
    mh = m2 / float(f32(1) - b1f ** step)
    vh = v2 / float(f32(1) - b2f ** step)
    p2 = np.asarray(param, np.float64) - float(f32(lr)) * mh / (np.sqrt(vh) + float(f32(eps)))
    return p2, m2, v2


__all__ = ["window", "ssim_map", "l1_dssim", "constant_ssim", "adam", "math"]
