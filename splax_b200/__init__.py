"""splax_b200: the splatting hot path of amacati/splax as sm_100a CUDA kernels.

Projection with the opacity-aware tile intersection, the intersection sort and tile-bin build,
and the forward and recompute-style backward blends run in libsplax_b200 (hand-written CUDA
behind a C ABI, include/splax_b200.h). This package mirrors the reference's public API
(splax/__init__.py:30-47) over torch tensors: ``render`` and ``render_log`` are differentiable
with torch.autograd with respect to the gaussian parameters, the camera pose and per-object
rigid transforms. ``mse_loss`` and ``l1_dssim_loss`` are fused loss-and-gradient kernels
for the training step around the render; ``Adam`` is its fused optimiser update;
``load_ply`` streams a 3DGS scene file onto the GPU. There is no CPU fallback.
"""

__version__ = "0.1.0"

from splax_b200 import utils
from splax_b200._cache import clear_cache, scratch_info
from splax_b200._io import load_ply, write_ply
from splax_b200._loss import l1_dssim_loss, mse_loss
from splax_b200._optim import Adam
from splax_b200._project import opacity_compensation, project, transform_ids
from splax_b200._rasterize import rasterize, rasterize_depth
from splax_b200._render import render, render_log

__all__ = [
    "Adam",
    "clear_cache",
    "l1_dssim_loss",
    "load_ply",
    "mse_loss",
    "opacity_compensation",
    "project",
    "rasterize",
    "rasterize_depth",
    "render",
    "render_log",
    "scratch_info",
    "transform_ids",
    "utils",
    "write_ply",
]
