"""Antialiased mode with the opacity compensation folded into the projection kernels.

The kernel's rho must equal the reference formula (``opacity_compensation``, the torch
restatement of splax/_project/_project.py:95-117) bit for bit -- both evaluate the same fp32
operations in the same order -- and an antialiased render's gradients must match the same
render taken through the torch formula (relative L2 <= 1e-4: only the rounding of the chained
conic cotangent differs)."""

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
