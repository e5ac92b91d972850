"""The training-step kernels around the render (config 3): the fused L1 + D-SSIM loss and the
fused Adam, against the CPU restatement in oracle/ssim.py (float64). Bars: loss relative error
<= 2e-5; gradient relative L2 <= 1e-4 (fp32 window sums against float64); Adam parameters and
moments relative error <= 1e-5 over three steps. The oracle itself is pinned by known answers
(identical images, constant images in closed form, the window's normalisation)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ssim as orc


def test_oracle_known_answers():
    rng = np.random.default_rng(1)
    a = rng.uniform(size=(2, 24, 31, 3))
    loss, grad = orc.l1_dssim(a, a)
    assert loss == 0.0
    c = np.full((1, 16, 16, 3), 0.3)
    d = np.full((1, 16, 16, 3), 0.6)
    s = float(orc.ssim_map(torch.tensor(c[0]), torch.tensor(d[0])).mean())
    assert abs(s - orc.constant_ssim(0.3, 0.6)) < 1e-12
    w = orc.window()
    assert abs(w.sum() - 1.0) < 1e-15 and np.allclose(w, w[::-1]) and w.argmax() == 5
    # lambda = 0 is the plain mean absolute error
    b = rng.uniform(size=(2, 24, 31, 3))
    l1, _ = orc.l1_dssim(a, b, ssim_lambda=0.0)
    assert abs(l1 - np.abs(a - b).mean()) < 1e-12


def test_oracle_adam_first_step_is_sign_step():
    # after one step the bias-corrected update is lr * g / (|g| + eps)
    g = np.array([0.5, -2.0, 1e-3])
    p, m, v = orc.adam(np.zeros(3), g, np.zeros(3), np.zeros(3), 1, lr=0.1)
    assert np.allclose(p, -0.1 * g / (np.abs(g) + 1e-8), rtol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,W", [(2, 48, 70), (1, 11, 11), (3, 37, 45)])
def test_l1_dssim_matches_oracle(B, H, W):
    import splax_b200 as sx
    rng = np.random.default_rng(B * 1000 + H)
    a = rng.uniform(size=(B, H, W, 3)).astype(np.float32)
    b = np.clip(a + rng.normal(0, 0.2, size=a.shape), 0, 1).astype(np.float32)
    ref_loss, ref_grad = orc.l1_dssim(a, b, 0.2)
    img = torch.tensor(a, device="cuda", requires_grad=True)
    tgt = torch.tensor(b, device="cuda")
    loss = sx.l1_dssim_loss(img, tgt, ssim_lambda=0.2)
    assert abs(loss.item() - ref_loss) <= 2e-5 * abs(ref_loss)
    (3.0 * loss).backward()
    g = img.grad.double().cpu().numpy()
    rel = np.linalg.norm(g - 3.0 * ref_grad) / np.linalg.norm(3.0 * ref_grad)
    assert rel <= 1e-4, rel


@pytest.mark.gpu
def test_l1_dssim_fused_pass_equals_separate_passes():
    """The one-pass loss-and-gradient (taken when the image requires grad) agrees with the
    separate loss and gradient entry points."""
    import ctypes

    import splax_b200 as sx
    from splax_b200 import _lib
    rng = np.random.default_rng(5)
    a = rng.uniform(size=(2, 61, 83, 3)).astype(np.float32)
    b = np.clip(a + rng.normal(0, 0.1, size=a.shape), 0, 1).astype(np.float32)
    img = torch.tensor(a, device="cuda", requires_grad=True)
    tgt = torch.tensor(b, device="cuda")
    loss_f = sx.l1_dssim_loss(img, tgt)
    (2.5 * loss_f).backward()
    with torch.no_grad():
        loss_s = sx.l1_dssim_loss(img, tgt)
    assert abs(loss_f.item() - loss_s.item()) <= 1e-6 * abs(loss_s.item())
    x = img.detach().contiguous()
    g = torch.empty_like(x)
    v = torch.tensor(2.5, device="cuda")
    lib = _lib.load()
    _lib.check(lib.splax_l1_dssim_loss_bwd(_lib.ptr(x), _lib.ptr(tgt), 2, 61, 83, 2,
                                           ctypes.c_float(0.2), _lib.ptr(v), _lib.ptr(g),
                                           _lib.stream_of(x)))
    rel = (img.grad - g).norm() / g.norm()
    assert rel.item() <= 1e-6, rel.item()
    # a retained graph runs the backward twice: the gradient accumulates, unchanged per call
    img.grad = None
    loss2 = sx.l1_dssim_loss(img, tgt)
    (2.5 * loss2).backward(retain_graph=True)
    first = img.grad.clone()
    (2.5 * loss2).backward()
    assert torch.allclose(img.grad, 2.0 * first, rtol=1e-6, atol=0.0)


@pytest.mark.gpu
def test_l1_dssim_shares_add_up_and_single_view():
    import splax_b200 as sx
    rng = np.random.default_rng(9)
    a = torch.tensor(rng.uniform(size=(4, 40, 52, 3)).astype(np.float32), device="cuda")
    b = torch.tensor(rng.uniform(size=(4, 40, 52, 3)).astype(np.float32), device="cuda")
    whole = sx.l1_dssim_loss(a, b).item()
    parts = (sx.l1_dssim_loss(a[:2], b[:2], views_total=4).item() +
             sx.l1_dssim_loss(a[2:], b[2:], views_total=4).item())
    assert abs(whole - parts) <= 1e-6 * abs(whole)
    one = sx.l1_dssim_loss(a[0], b[0]).item()
    ref, _ = orc.l1_dssim(a[:1].cpu().numpy(), b[:1].cpu().numpy())
    assert abs(one - ref) <= 2e-5 * abs(ref)
    for _ in range(2):  # deterministic
        assert sx.l1_dssim_loss(a, b).item() == whole


@pytest.mark.gpu
def test_adam_matches_optax_restatement():
    import splax_b200 as sx
    rng = np.random.default_rng(4)
    shapes = [(1001, 3), (7,), (256, 4)]
    lrs = [1e-3, 5e-2, 2e-4]
    p0 = [rng.normal(size=s).astype(np.float32) for s in shapes]
    params = [torch.tensor(x, device="cuda") for x in p0]
    opt = sx.Adam(params, lrs)
    ref = [(x.astype(np.float64), np.zeros(x.shape), np.zeros(x.shape)) for x in p0]
    for step in range(1, 4):
        grads = [rng.normal(size=s).astype(np.float32) for s in shapes]
        opt.step([torch.tensor(g, device="cuda") for g in grads])
        ref = [orc.adam(p, g, m, v, step, lr) for (p, m, v), g, lr in zip(ref, grads, lrs)]
    for t, m, v, (rp, rm, rv) in zip(params, opt.exp_avg, opt.exp_avg_sq, ref):
        for got, want in ((t, rp), (m, rm), (v, rv)):
            got = got.double().cpu().numpy()
            assert np.abs(got - want).max() <= 1e-5 * max(np.abs(want).max(), 1e-3)
