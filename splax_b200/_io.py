"""3DGS .ply scenes (splax/io.py:78-132): ``load_ply`` reads a file straight into device tensors
through the library's streaming loader; ``write_ply`` writes render-space splats in the layout
the reference's ``write_ply`` produces (host side, numpy)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from splax_b200 import _lib

_C0 = 0.28209479177387814  # degree-0 SH basis constant: colors = f_dc * C0 + 0.5
_FIELDS = (["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2", "opacity"]
           + [f"scale_{i}" for i in range(3)] + [f"rot_{i}" for i in range(4)])


def load_ply(path: str | Path, device: torch.device | str | None = None):
    """Read a 3DGS ``.ply`` into means, scales (N, 3), quats wxyz (N, 4), colors (N, 3) and
    opacities (N, 1) fp32 tensors on a CUDA device, decoding exp / normalisation / SH-DC /
    sigmoid on the GPU as splax.io.load_ply does on the host."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else \
        torch.device(device)
    if dev.type != "cuda":
        raise ValueError("splax_b200 loads .ply files onto CUDA devices only")
    lib = _lib.load()
    p = str(Path(path)).encode()
    n = _lib.ctypes.c_int64(0)
    _lib.check(lib.splax_ply_info(p, _lib.ctypes.byref(n)))
    N = int(n.value)
    f32 = dict(device=dev, dtype=torch.float32)
    means, scales = torch.empty((N, 3), **f32), torch.empty((N, 3), **f32)
    quats, colors = torch.empty((N, 4), **f32), torch.empty((N, 3), **f32)
    opac = torch.empty((N, 1), **f32)
    with torch.cuda.device(dev):
        rc = lib.splax_ply_load(p, N, _lib.ptr(means), _lib.ptr(scales), _lib.ptr(quats),
                                _lib.ptr(colors), _lib.ptr(opac), _lib.stream_of(means))
    _lib.check(rc)
    return means, scales, quats, colors, opac


def write_ply(path: str | Path, means, scales, quats, colors, opacities) -> None:
    """Write render-space splats (means (N,3), positive scales (N,3), wxyz quats (N,4), RGB
    colors in [0,1] (N,3), opacities in [0,1]) as a binary little-endian 3DGS ``.ply`` with the
    reference's fields and order (splax/io.py:101-132)."""
    from scipy.special import logit

    def host(x):
        if isinstance(x, torch.Tensor):
            x = x.detach().cpu().numpy()
        return np.asarray(x, np.float32)

    means, scales, quats, colors, opacities = map(host, (means, scales, quats, colors, opacities))
    quats = quats / np.linalg.norm(quats, axis=-1, keepdims=True)
    f_dc = (colors - 0.5) / _C0
    opac_logit = logit(np.clip(opacities.reshape(-1, 1), 1e-7, 1.0 - 1e-7))
    n = means.shape[0]
    data = np.hstack([means, np.zeros((n, 3)), f_dc, opac_logit, np.log(scales), quats])
    verts = np.empty(n, dtype=[(f, "<f4") for f in _FIELDS])
    for field, column in zip(_FIELDS, data.T, strict=True):
        verts[field] = column
    header = ("ply\nformat binary_little_endian 1.0\n" f"element vertex {n}\n"
              + "".join(f"property float {f}\n" for f in _FIELDS) + "end_header\n")
    with open(path, "wb") as fh:
        fh.write(header.encode("ascii"))
        fh.write(verts.tobytes())
