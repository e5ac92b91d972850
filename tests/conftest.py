"""Shared pytest configuration: the ``gpu`` marker and seeded synthetic scenes."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")


def random_scene(n: int, seed: int = 0, *, spread: float = 0.5, smin: float = 0.02,
                 smax: float = 0.08, omin: float = 0.1, omax: float = 0.6):
    """Scene like the reference tests' _scene (tests/test_warp_grad.py:46-59), numpy-seeded.

    Returns means (n,3), scales (n,3), quats wxyz (n,4), colors (n,3), opacities (n,), bg (3,).
    """
    rng = np.random.default_rng(seed)
    means = (rng.normal(size=(n, 3)) * spread).astype(np.float32)
    scales = rng.uniform(smin, smax, size=(n, 3)).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    quats /= np.linalg.norm(quats, axis=-1, keepdims=True)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    opac = rng.uniform(omin, omax, size=n).astype(np.float32)
    bg = rng.uniform(size=3).astype(np.float32)
    return means, scales, quats, colors, opac, bg


def viewmat(dx: float = 0.2, dy: float = -0.1, dz: float = 5.0) -> np.ndarray:
    return np.array([[1, 0, 0, dx], [0, 1, 0, dy], [0, 0, 1, dz], [0, 0, 0, 1]], np.float32)


def cam(H: int, W: int) -> dict:
    """Camera statics as in the reference tests' _pk (tests/test_warp_grad.py:70-77)."""
    return {"img_shape": (H, W), "f": (float(H), float(H)), "c": (W // 2, H // 2)}


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle
