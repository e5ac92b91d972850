"""Device .ply loading (splax/io.py:78-132) against the CPU restatement in oracle/ply.py, which
parses the records with a numpy structured dtype. Bars: means and colors exact up to 1 ulp of
the fused multiply-add; scales, quats, opacities within 2e-7 relative (the GPU's expf / division
vs numpy's). Header errors are refused on the CPU."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import ply as orc
from splax_b200 import _io, _lib


def _splats(n, seed=0):
    rng = np.random.default_rng(seed)
    means = rng.normal(size=(n, 3)).astype(np.float32)
    scales = np.exp(rng.normal(-3, 0.5, size=(n, 3))).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    opac = rng.uniform(0.01, 0.99, size=(n,)).astype(np.float32)
    return means, scales, quats, colors, opac


def _info(path):
    lib = _lib.load()
    n = ctypes.c_int64(-1)
    rc = lib.splax_ply_info(str(path).encode(), ctypes.byref(n))
    return rc, n.value


def _odd_layout(path, n, seed=1):
    """INRIA-style record with extra properties, a uchar that misaligns the floats, and the
    needed fields in another order."""
    rng = np.random.default_rng(seed)
    fields = [("x", "<f4"), ("y", "<f4"), ("z", "<f4"), ("flag", "u1"), ("nx", "<f4"),
              ("ny", "<f4"), ("nz", "<f4"), ("f_dc_0", "<f4"), ("f_dc_1", "<f4"),
              ("f_dc_2", "<f4")] + [(f"f_rest_{i}", "<f4") for i in range(9)] + [
        ("opacity", "<f4"), ("rot_0", "<f4"), ("rot_1", "<f4"), ("rot_2", "<f4"),
        ("rot_3", "<f4"), ("scale_0", "<f4"), ("scale_1", "<f4"), ("scale_2", "<f4"),
        ("w", "<f8")]
    v = np.zeros(n, dtype=fields)
    for name, t in fields:
        v[name] = rng.normal(size=n).astype(t)
    names = {"u1": "uchar", "<f4": "float", "<f8": "double"}
    header = (f"ply\nformat binary_little_endian 1.0\ncomment odd layout\nelement vertex {n}\n"
              + "".join(f"property {names[t]} {name}\n" for name, t in fields)
              + "element face 0\nproperty list uchar int vertex_indices\nend_header\n")
    with open(path, "wb") as fh:
        fh.write(header.encode())
        fh.write(v.tobytes())


def test_info_reads_counts(tmp_path):
    p = tmp_path / "a.ply"
    _io.write_ply(p, *_splats(123))
    assert _info(p) == (0, 123)
    p2 = tmp_path / "b.ply"
    _odd_layout(p2, 77)
    assert _info(p2) == (0, 77)


@pytest.mark.parametrize("header,msg", [
    ("ply\nformat ascii 1.0\nelement vertex 1\nproperty float x\nend_header\n", "format"),
    ("ply\nformat binary_little_endian 1.0\nelement vertex 1\nproperty float x\nend_header\n",
     "lacks the field"),
    ("ply\nformat binary_little_endian 1.0\nelement vertex 1\nproperty list uchar int x\n"
     "end_header\n", "list"),
    ("not a ply\n", "not a PLY"),
])
def test_info_refuses_bad_headers(tmp_path, header, msg):
    p = tmp_path / "bad.ply"
    p.write_bytes(header.encode())
    rc, _ = _info(p)
    assert rc == 1 and msg in _lib.load().splax_last_error().decode()


def test_oracle_round_trips_the_writer(tmp_path):
    m, s, q, c, o = _splats(50)
    p = tmp_path / "r.ply"
    _io.write_ply(p, m, s, q, c, o)
    means, scales, quats, colors, opac = orc.load_ply(p)
    assert np.array_equal(means, m)
    assert np.allclose(scales, s, rtol=1e-6)
    assert np.allclose(quats, q / np.linalg.norm(q, axis=-1, keepdims=True), atol=1e-7)
    assert np.allclose(colors, c, atol=1e-6) and np.allclose(opac[:, 0], o, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["reference", "odd"])
def test_device_load_matches_oracle(tmp_path, layout):
    import splax_b200 as sx
    p = tmp_path / "s.ply"
    n = 100_003
    if layout == "reference":
        _io.write_ply(p, *_splats(n))
    else:
        _odd_layout(p, n)
    got = [t.cpu().numpy() for t in sx.load_ply(p)]
    want = orc.load_ply(p)
    for name, g, w in zip(("means", "scales", "quats", "colors", "opac"), got, want):
        assert g.shape == w.shape, name
        if name == "means":
            assert np.array_equal(g, w)
        elif name == "colors":
            assert np.abs(g - w).max() <= 6e-8, name
        else:
            assert np.abs(g - w).max() <= 2e-7 * max(1.0, np.abs(w).max()), name


@pytest.mark.gpu
def test_device_load_refuses_truncated_file(tmp_path):
    import splax_b200 as sx
    p = tmp_path / "t.ply"
    _io.write_ply(p, *_splats(1000))
    raw = p.read_bytes()
    p.write_bytes(raw[:-100])
    with pytest.raises(ValueError, match="shorter"):
        sx.load_ply(p)
