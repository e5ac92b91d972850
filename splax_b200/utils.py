"""Camera helpers and the seeded synthetic scenes of the benchmark configurations.

``look_at`` follows splax/utils.py:9-30 (OpenCV world-to-camera, x right, y down). The scene
builders generate the seeded inputs of each benchmark configuration (0-4), in a fixed order
with numpy's default_rng, so the CUDA path and the CPU baseline consume identical bytes.
"""

from __future__ import annotations

import numpy as np


def look_at(eye, target, up=(0.0, 1.0, 0.0)) -> np.ndarray:
    """(..., 4, 4) float32 world-to-camera matrices looking from ``eye`` to ``target``."""
    eye = np.asarray(eye, np.float64)
    target = np.asarray(target, np.float64)
    z = target - eye
    norm = np.linalg.norm(z, axis=-1, keepdims=True)
    assert (norm > 0).all(), "eye and target must differ"
    z = z / norm
    x = np.cross(z, np.asarray(up, np.float64))
    x = x / np.linalg.norm(x, axis=-1, keepdims=True)
    y = np.cross(z, x)
    R = np.stack([x, y, z], axis=-1)  # camera-to-world rotation, columns x, y, z
    Rt = np.swapaxes(R, -1, -2)
    w2c = np.zeros((*z.shape[:-1], 4, 4))
    w2c[..., :3, :3] = Rt
    w2c[..., :3, 3] = -np.einsum("...ij,...j->...i", Rt, eye)
    w2c[..., 3, 3] = 1.0
    return w2c.astype(np.float32)


def _gaussians(rng, n, means, log_scale_mu, log_scale_sigma, opac_mu):
    scales = np.exp(rng.normal(log_scale_mu, log_scale_sigma, size=(n, 3))).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    quats /= np.linalg.norm(quats, axis=-1, keepdims=True)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-rng.normal(opac_mu, 1.0, size=n)))).astype(np.float32)
    return means.astype(np.float32), scales, quats, colors, opac


CONFIGS = {
    0: dict(n=10_000, H=256, W=256, f=300.0, B=1),
    1: dict(n=200_000, H=800, W=800, f=1100.0, B=1),
    2: dict(n=1_000_000, H=1080, W=1920, f=1400.0, B=8),
    3: dict(n=3_000_000, H=840, W=1297, f=1150.0, B=32),
    4: dict(n=6_000_000, H=2160, W=3840, f=2800.0, B=64),
}


def synthetic_scene(config: int, seed: int = 0, n: int | None = None) -> dict:
    """Seeded inputs of one benchmark configuration: gaussians (means, scales, wxyz quats,
    colors, opacities), the camera stack, image size, focal length and a target image stack."""
    cfg = dict(CONFIGS[config])
    if n is not None:
        cfg["n"] = n
    rng = np.random.default_rng(seed)
    N = cfg["n"]
    if config == 0:
        means = rng.uniform(-1, 1, size=(N, 3))
        g = _gaussians(rng, N, means, -4.0, 0.5, 0.0)
        views = look_at(np.array([[0.0, 0.0, 4.0]]), np.zeros(3))
    elif config == 1:
        means = rng.uniform(-2, 2, size=(N, 3))
        g = _gaussians(rng, N, means, -4.0, 0.5, 0.0)
        views = look_at(np.array([[0.0, 0.0, 6.0]]), np.zeros(3))
    elif config == 2:
        means = rng.normal(0.0, 1.5, size=(N, 3))
        g = _gaussians(rng, N, means, -4.0, 0.5, 0.0)
        phi = 2 * np.pi * np.arange(cfg["B"]) / cfg["B"]
        eyes = np.stack([5 * np.cos(phi), np.ones_like(phi), 5 * np.sin(phi)], -1)
        views = look_at(eyes, np.zeros(3))
    elif config == 3:
        means = rng.normal(0.0, 3.0, size=(N, 3))
        g = _gaussians(rng, N, means, -4.0, 0.5, 0.0)
        d = rng.normal(size=(cfg["B"], 3))
        d[:, 1] = np.abs(d[:, 1]) + 0.05
        d /= np.linalg.norm(d, axis=-1, keepdims=True)
        views = look_at(6.0 * d, np.zeros(3))
    else:
        means = rng.normal(0.0, 4.0, size=(N, 3))
        g = _gaussians(rng, N, means, -3.5, 0.7, 1.0)
        dirs = []
        while len(dirs) < cfg["B"]:
            v = rng.normal(size=3)
            v /= np.linalg.norm(v)
            if abs(v[1]) <= 0.99:
                dirs.append(v)
        views = look_at(8.0 * np.array(dirs), np.zeros(3))
    target = None
    means, scales, quats, colors, opac = g
    return dict(means=means, scales=scales, quats=quats, colors=colors, opacities=opac,
                viewmats=views, H=cfg["H"], W=cfg["W"], f=cfg["f"], B=views.shape[0],
                background=np.ones(3, np.float32) if config == 0 else np.zeros(3, np.float32),
                target_seed=seed + 1, target=target)


def target_images(scene: dict, cams=None) -> np.ndarray:
    """Seeded uniform-[0,1] targets (len(cams), H, W, 3) for the MSE / L1 losses; camera k's
    image depends on (target_seed, k) only, so a rank can make just the cameras it renders."""
    ks = range(scene["B"]) if cams is None else cams
    out = np.empty((len(ks), scene["H"], scene["W"], 3), np.float32)
    for i, k in enumerate(ks):
        rng = np.random.default_rng((scene["target_seed"], k))
        out[i] = rng.uniform(size=(scene["H"], scene["W"], 3))
    return out
