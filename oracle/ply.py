"""CPU restatement of splax.io.load_ply (splax/io.py:78-98), for tests only: the vertex records
are parsed with a numpy structured dtype built from the header (independently of the library's
C parser) and decoded in float32 numpy exactly as the reference's formulas read:
means, exp(scale), rot / |rot|, clip(f_dc * C0 + 0.5, 0, 1), sigmoid(opacity)."""

from __future__ import annotations

import numpy as np

C0 = np.float32(0.28209479177387814)
_TYPES = {"char": "i1", "uchar": "u1", "int8": "i1", "uint8": "u1", "short": "<i2",
          "ushort": "<u2", "int16": "<i2", "uint16": "<u2", "int": "<i4", "uint": "<u4",
          "int32": "<i4", "uint32": "<u4", "float": "<f4", "float32": "<f4", "double": "<f8",
          "float64": "<f8"}


def read_vertices(path) -> np.ndarray:
    raw = open(path, "rb").read()
    end = raw.index(b"end_header\n") + len(b"end_header\n")
    lines = raw[:end].decode("ascii").splitlines()
    assert lines[0] == "ply" and "binary_little_endian" in lines[1]
    fields, n, in_v = [], None, False
    for ln in lines:
        t = ln.split()
        if t[0] == "element":
            in_v = t[1] == "vertex"
            if in_v:
                n = int(t[2])
        elif t[0] == "property" and in_v:
            fields.append((t[2], _TYPES[t[1]]))
    return np.frombuffer(raw, dtype=np.dtype(fields), count=n, offset=end)


def load_ply(path):
    v = read_vertices(path)
    f = lambda *names: np.stack([v[k].astype(np.float32) for k in names], -1)  # noqa: E731
    means = f("x", "y", "z")
    scales = np.exp(f("scale_0", "scale_1", "scale_2"))
    q = f("rot_0", "rot_1", "rot_2", "rot_3")
    quats = q / np.linalg.norm(q, axis=-1, keepdims=True)
    colors = np.clip(f("f_dc_0", "f_dc_1", "f_dc_2") * C0 + np.float32(0.5), 0.0, 1.0)
    o = v["opacity"].astype(np.float32)
    opac = (np.float32(1) / (np.float32(1) + np.exp(-o)))[:, None]
    return means, scales, quats, colors, opac
