"""Rendering entry point (splax/_render.py): project, optional antialiasing, rasterize."""

from __future__ import annotations

from collections.abc import Sequence

import torch

from splax_b200._project import project, transform_ids
from splax_b200._rasterize import rasterize, rasterize_depth

_AA_EPS = 0.3  # the projection's screen-space dilation (splax/_project/_project.py:95)


def render(
    means3d: torch.Tensor,
    scales: torch.Tensor,
    quats: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    *,
    viewmat: torch.Tensor,
    background: torch.Tensor,
    img_shape: tuple[int, int],
    f: tuple[float, float],
    c: tuple[float, float] | None = None,
    glob_scale: float = 1.0,
    clip_thresh: float = 0.01,
    antialiased: bool = False,
    render_depth: bool = False,
    gaussian_transforms: torch.Tensor | None = None,
    gaussian_slices: Sequence[tuple[int, int]] | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Render a splat (splax/_render.py:29-115); differentiable through torch.autograd.

    means3d (N,3), scales (N,3), quats wxyz (N,4), colors (N,3), opacities (N,) or (N,1),
    viewmat (4,4) world-to-camera, background (3,). A leading batch axis B on any of them (a
    (B,4,4) viewmat stack for B cameras) renders all B images in one launch, returning
    (B,H,W,3). Slices of gaussians may follow rigid transforms (K,4,4). Returns the image and,
    with ``render_depth``, the expected depth map (else None).
    """
    if (gaussian_transforms is None) != (gaussian_slices is None):
        raise ValueError("gaussian_transforms and gaussian_slices must be passed together")
    tf_ids = None
    if gaussian_transforms is not None and gaussian_slices is not None:
        if tuple(gaussian_transforms.shape[-3:]) != (len(gaussian_slices), 4, 4):
            raise ValueError(
                f"gaussian_transforms shape {tuple(gaussian_transforms.shape)} does not "
                f"match {len(gaussian_slices)} slices, expected (K, 4, 4)")
        tf_ids = transform_ids(means3d.shape[-2], gaussian_slices, device=means3d.device)

    outs = project(
        means3d, scales, quats, viewmat, opacities=opacities, img_shape=img_shape, f=f, c=c,
        glob_scale=glob_scale, clip_thresh=clip_thresh, gaussian_transforms=gaussian_transforms,
        transform_ids=tf_ids, antialias_eps=_AA_EPS if antialiased else None)
    xys, depths, radii, conics, _, cum_tiles_hit = outs[:6]

    blend_opacities = opacities
    map_opacities = None
    if antialiased:
        # opacity_compensation(conics, radii), computed by the projection kernel
        rho = outs[6]
        n = means3d.shape[-2]
        lead = rho.shape[:-1]
        blend_opacities = opacities.reshape(*([1] * len(lead)), n) * rho if lead else \
            opacities.reshape(n) * rho
        map_opacities = opacities  # the tile intersection stays on the raw opacity

    inputs = (colors, blend_opacities, background, xys, depths, radii, conics, cum_tiles_hit)
    if render_depth:
        return rasterize_depth(*inputs, img_shape=img_shape, map_opacities=map_opacities)
    return rasterize(*inputs, img_shape=img_shape, map_opacities=map_opacities), None


def render_log(
    means3d: torch.Tensor,
    log_scales: torch.Tensor,
    quats: torch.Tensor,
    logit_colors: torch.Tensor,
    logit_opacities: torch.Tensor,
    *,
    viewmat: torch.Tensor,
    background: torch.Tensor,
    img_shape: tuple[int, int],
    f: tuple[float, float],
    c: tuple[float, float] | None = None,
    glob_scale: float = 1.0,
    clip_thresh: float = 0.01,
    antialiased: bool = False,
    render_depth: bool = False,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Render from the log / logit training parameterisation (splax/_render.py:118-168)."""
    scales = torch.exp(log_scales)
    quats = quats / (torch.linalg.norm(quats, dim=-1, keepdim=True) + 1e-8)
    colors = torch.sigmoid(logit_colors)
    opacities = torch.sigmoid(logit_opacities)
    return render(means3d, scales, quats, colors, opacities, viewmat=viewmat,
                  background=background, img_shape=img_shape, f=f, c=c, glob_scale=glob_scale,
                  clip_thresh=clip_thresh, antialiased=antialiased, render_depth=render_depth)
