"""Fused MSE loss: the value and gradient against plain torch fp32 (bars: loss relative error
<= 1e-5 with fp64 as the yardstick, gradient max-abs error <= 1e-6 relative to its scale),
the vector and scalar paths, an empty input and the CPU refusal."""

from __future__ import annotations

import pytest
import torch

import splax_b200 as sx


def test_mse_loss_refuses_cpu_tensors():
    a = torch.zeros(8)
    with pytest.raises(ValueError, match="CUDA"):
        sx.mse_loss(a, a)


def test_mse_loss_rejects_bad_denom():
    a = torch.zeros(0)
    with pytest.raises(ValueError, match="denom"):
        sx.mse_loss(a, a)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,offset", [((8, 108, 192, 3), 0), ((1001, 3), 0), ((4099,), 1)])
def test_mse_loss_matches_torch(shape, offset):
    g = torch.Generator(device="cuda").manual_seed(3)
    n = torch.Size(shape).numel()
    # offset 1 makes both pointers 4 bytes past a 16-byte boundary: the scalar path
    base_a = torch.rand(n + offset, device="cuda", generator=g)
    base_t = torch.rand(n + offset, device="cuda", generator=g)
    img = base_a[offset:].view(shape).clone().requires_grad_() if offset == 0 else \
        base_a[offset:].view(shape).requires_grad_()
    tgt = base_t[offset:].view(shape)
    denom = 3.0 * n
    loss = sx.mse_loss(img, tgt, denom=denom)
    ref64 = ((img.detach().double() - tgt.double()) ** 2).sum() / denom
    assert abs(loss.item() - ref64.item()) <= 1e-5 * abs(ref64.item())
    (2.5 * loss).backward()
    ref_grad = 2.5 * 2.0 * (img.detach() - tgt) / denom
    scale = ref_grad.abs().max().item()
    assert (img.grad - ref_grad).abs().max().item() <= 1e-6 * scale


@pytest.mark.gpu
def test_mse_loss_is_deterministic_and_handles_empty():
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.rand(3_000_001, device="cuda", generator=g)
    t = torch.rand(3_000_001, device="cuda", generator=g)
    first = sx.mse_loss(a, t)
    for _ in range(3):
        assert torch.equal(sx.mse_loss(a, t), first)
    e = torch.empty(0, device="cuda")
    assert sx.mse_loss(e, e, denom=1.0).item() == 0.0
