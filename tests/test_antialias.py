"""Antialiased mode with the opacity compensation folded into the projection kernels.

The kernel's rho must equal the reference formula (``opacity_compensation``, the torch
restatement of splax/_project/_project.py:95-117) bit for bit -- both evaluate the same fp32
operations in the same order -- and an antialiased render's gradients must match the same
render taken through the torch formula (relative L2 <= 1e-4: only the rounding of the chained
conic cotangent differs). Against the C oracle, an antialiased render (splax/_render.py:103-107:
blend opacities opacity * rho, tile intersection on the raw opacity) must give the image within
max-abs 1e-4 on the pixels whose threshold decisions the oracle does not flag, and the
gradients of all five arrays and the viewmat within relative L2 1e-3, with rho's vjp derived
independently on the CPU (tests/_oracle_chain.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import splax_b200 as sx
from splax_b200 import utils


def _scene(n=3000, seed=5, B=2):
    rng = np.random.default_rng(seed)
    means = rng.normal(0.0, 1.0, size=(n, 3)).astype(np.float32)
    scales = np.exp(rng.normal(-3.0, 0.5, size=(n, 3))).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    quats /= np.linalg.norm(quats, axis=-1, keepdims=True)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.0, size=n)))).astype(np.float32)
    phi = np.linspace(0, 1.2, B)
    eyes = np.stack([4 * np.cos(phi), 0.5 * np.ones_like(phi), 4 * np.sin(phi)], -1)
    views = utils.look_at(eyes, np.zeros(3)).astype(np.float32)
    t = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    return [t(means), t(scales), t(quats), t(colors), t(opac)], t(views)


@pytest.mark.gpu
def test_kernel_rho_matches_formula_bitwise():
    params, views = _scene()
    out = sx.project(params[0], params[1], params[2], views, opacities=params[4],
                     img_shape=(120, 160), f=(150.0, 150.0), antialias_eps=0.3)
    xys, depths, radii, conics, nth, cum, rho = out
    ref = sx.opacity_compensation(conics, radii)
    assert rho.shape == ref.shape
    assert torch.equal(rho, ref)
    assert (rho[radii.squeeze(-1) <= 0] == 1.0).all()
    assert ((rho > 0) & (rho <= 1)).all()


def _grads(params, views, fold: bool):
    ps = [p.clone().requires_grad_() for p in params]
    bg = torch.tensor([0.2, 0.3, 0.4], device="cuda")
    kw = dict(background=bg, img_shape=(120, 160), f=(150.0, 150.0))
    if fold:
        img, _ = sx.render(*ps, viewmat=views, antialiased=True, **kw)
    else:
        out = sx.project(ps[0], ps[1], ps[2], views, opacities=ps[4], img_shape=kw["img_shape"],
                         f=kw["f"])
        xys, depths, radii, conics, _, cum = out
        rho = sx.opacity_compensation(conics, radii)
        blend = ps[4].reshape(1, -1) * rho
        img = sx.rasterize(ps[3], blend, bg, xys, depths, radii, conics, cum,
                           img_shape=kw["img_shape"], map_opacities=ps[4])
    g = torch.Generator(device="cuda").manual_seed(7)
    w = torch.rand(img.shape, device="cuda", generator=g)
    (img * w).sum().backward()
    return img.detach(), [p.grad for p in ps]


@pytest.mark.gpu
def test_antialiased_render_matches_torch_formula():
    params, views = _scene()
    img_a, g_a = _grads(params, views, fold=True)
    img_b, g_b = _grads(params, views, fold=False)
    assert torch.equal(img_a, img_b)
    for name, a, b in zip(("means", "scales", "quats", "colors", "opacities"), g_a, g_b):
        rel = ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
        assert rel <= 1e-4, (name, rel)


@pytest.mark.gpu
def test_antialiased_render_vs_oracle(oracle_lib):
    """End to end with antialiased=True: the CUDA path (rho and its cotangent folded into the
    projection kernels) against the oracle's projection, fp32 rho, blend and the float64 vjp
    chain; the image cotangent is zero on pixels the oracle flags as threshold ties."""
    import _oracle_chain as ch
    from conftest import cam, random_scene, viewmat

    n, H, W, eps = 3000, 128, 128, 0.3
    m, s, q, c, op, bg = random_scene(n, 21, smin=0.005, smax=0.05)
    vm = viewmat()
    ref_img, _, st = ch.render(m, s, q, c, op, bg, vm, antialias_eps=eps, **cam(H, W))
    flags = st["flags"].reshape(H, W)
    assert (flags == 0).mean() > 0.99
    rho = st["rho"][np.asarray(st["radii"]).reshape(-1) > 0]
    assert rho.min() < 0.99  # the compensation is active on part of the scene
    w = np.random.default_rng(4).uniform(size=(H, W, 3)).astype(np.float32) / (H * W)
    w[flags != 0] = 0.0
    t = lambda a: torch.tensor(np.ascontiguousarray(a), device="cuda")  # noqa: E731
    params = [t(x).requires_grad_() for x in (m, s, q, c, op)]
    vm_t = t(vm).requires_grad_()
    img, _ = sx.render(*params, viewmat=vm_t, background=t(bg), antialiased=True, **cam(H, W))
    diff = np.abs(img.detach().cpu().numpy() - ref_img).max(axis=-1)
    assert diff[flags == 0].max() <= 1e-4
    (img * t(w)).sum().backward()
    ref = ch.grads(m, s, q, c, op, bg, vm, w, antialias_eps=eps, **cam(H, W))

    def rel(a, b):
        a, b = np.asarray(a, np.float64).reshape(b.shape), np.asarray(b, np.float64)
        return np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30)

    names = ["means", "scales", "quats", "colors", "opacities"]
    errs = {k: rel(p.grad.cpu().numpy(), g) for k, p, g in zip(names, params, ref[:5])}
    errs["viewmat"] = rel(vm_t.grad.cpu().numpy(), ref[5])
    assert max(errs.values()) <= 1e-3, errs


def test_oracle_chain_compensation_matches_formula():
    """The oracle chain's fp32 rho2 (numpy) equals the torch restatement of the reference
    formula bit for bit on the CPU, its rho is the correctly rounded square root of the clipped
    rho2 (1 for culled entries; torch's vectorised CPU sqrt is not correctly rounded, the GPU's
    is), and its vjp agrees with torch autograd of the formula inside the clip."""
    import _oracle_chain as ch

    rng = np.random.default_rng(12)
    conics = np.abs(rng.normal(0.0, 1.5, size=(4000, 3))).astype(np.float32)
    conics[:, 1] = rng.normal(0.0, 0.3, size=4000).astype(np.float32)
    conics[:5] = [[0, 0, 0], [1e-6, 0, 1e-6], [20, 0, 20], [3.3333, 0, 0], [0, 0, 3.3333]]
    radii = rng.integers(-1, 5, size=4000).astype(np.int32)
    rho, rho2 = ch.compensation(conics, radii, 0.3)
    t = torch.tensor(conics)
    a, b, c = t[:, 0], t[:, 1], t[:, 2]
    assert np.array_equal(rho2, (1.0 - 0.3 * (a + c) + (0.3 * 0.3) * (a * c - b * b)).numpy())
    exact = np.sqrt(np.clip(rho2.astype(np.float64), 0.0, 1.0)).astype(np.float32)
    assert np.array_equal(rho, np.where(radii > 0, exact, np.float32(1.0)))
    ct = torch.tensor(conics, requires_grad=True)
    ref = sx.opacity_compensation(ct, torch.tensor(radii))
    v = rng.normal(size=4000)
    ref.backward(torch.tensor(v, dtype=torch.float32))
    mine = ch.compensation_vjp(conics, radii, 0.3, v)
    inside = (radii > 0) & (rho2 > 0) & (rho2 < 1)
    got, want = mine[inside], ct.grad.numpy()[inside].astype(np.float64)
    assert np.linalg.norm(got - want) <= 1e-6 * np.linalg.norm(want)
