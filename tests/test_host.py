"""CPU tests of the host side: the C ABI library's exports and the torch layer's logic.

No kernel runs here (there is no GPU in the build container); calls that would launch one are
not made.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import cam, random_scene, viewmat

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from splax_b200 import _build, _lib

    if not _build.up_to_date():
        _build.build()
    return _lib.load()


def _declared() -> list[str]:
    names = []
    for h in (ROOT / "include").glob("*.h"):
        names += re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(splax_\w+)\s*\(", h.read_text(), re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(lib):
    names = _declared()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name


def test_ctypes_signatures_cover_the_header(lib):
    from splax_b200 import _lib

    assert set(_declared()) == set(_lib.SIGNATURES)
    assert lib.splax_version().decode().startswith("splax_b200")


def test_header_argument_counts_match_ctypes():
    """Each ctypes signature has as many parameters as the C declaration."""
    from splax_b200 import _lib

    text = (ROOT / "include" / "splax_b200.h").read_text()
    for name, args in _lib.SIGNATURES.items():
        m = re.search(rf"^\s*(?:const\s+)?\w+\s*\*?\s*{name}\s*\(([^;]*?)\)\s*;", text,
                      re.S | re.M)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))


def test_errors_map_to_python_exceptions(lib):
    from splax_b200 import _lib

    with pytest.raises(ValueError):
        _lib.check(_lib.SPLAX_ERR_INVALID_ARGUMENT)
    with pytest.raises(ValueError):
        _lib.check(_lib.SPLAX_ERR_KEY_OVERFLOW)
    with pytest.raises(_lib.SplaxDeviceError):
        _lib.check(_lib.SPLAX_ERR_DEVICE)
    with pytest.raises(torch.cuda.OutOfMemoryError):
        _lib.check(_lib.SPLAX_ERR_OUT_OF_MEMORY)


def test_cpu_tensors_are_refused():
    """No CPU fallback: the torch layer refuses host tensors before any launch."""
    import splax_b200 as sx

    m, s, q, c, op, bg = random_scene(10, 0)
    with pytest.raises(ValueError, match="CUDA"):
        sx.render(*(torch.tensor(x) for x in (m, s, q, c, op)), viewmat=torch.tensor(viewmat()),
                  background=torch.tensor(bg), **cam(32, 32))


def test_key_width_rule_and_hook(monkeypatch):
    from splax_b200 import _sort

    assert _sort.key_bits_for(1, 1080, 1920) == 32
    assert _sort.key_bits_for(8, 1080, 1920) == 64  # 3 + 13 image/tile bits leave 15 < 16
    assert _sort.key_bits_for(4, 1080, 1920) == 32
    monkeypatch.setattr(_sort, "_use_32bit_keys", lambda depth_bits: False)
    assert _sort.key_bits_for(1, 64, 64) == 64
    with pytest.raises(ValueError, match="key overflow"):
        _sort.key_bits_for(1 << 20, 4096, 8192)


def test_transform_ids_validation():
    import splax_b200 as sx

    ids = sx.transform_ids(10, [(0, 3), (5, 8)])
    assert ids.tolist() == [0, 0, 0, -1, -1, 1, 1, 1, -1, -1]
    with pytest.raises(ValueError, match="outside"):
        sx.transform_ids(10, [(5, 11)])
    with pytest.raises(ValueError, match="overlap"):
        sx.transform_ids(10, [(0, 5), (4, 8)])


def test_render_argument_checks():
    import splax_b200 as sx

    z = torch.zeros((4, 3))
    with pytest.raises(ValueError, match="together"):
        sx.render(z, z, torch.zeros((4, 4)), z, torch.zeros(4), viewmat=torch.eye(4),
                  background=torch.zeros(3), img_shape=(8, 8), f=(8.0, 8.0),
                  gaussian_transforms=torch.zeros((1, 4, 4)))


def test_batch_size_inference():
    from splax_b200._project import batch_size

    n = 6
    shared = torch.zeros((n, 3)), torch.zeros((n, 3)), torch.zeros((n, 4))
    assert batch_size(n, *shared, torch.eye(4), torch.zeros(n)) == 0
    assert batch_size(n, *shared, torch.zeros((3, 4, 4)), torch.zeros(n)) == 3
    assert batch_size(n, torch.zeros((2, n, 3)), *shared[1:], torch.eye(4), torch.zeros(n)) == 2
    with pytest.raises(ValueError, match="inconsistent"):
        batch_size(n, torch.zeros((2, n, 3)), *shared[1:], torch.zeros((3, 4, 4)), torch.zeros(n))


def test_opacity_compensation_closed_form(oracle_lib):
    """rho from the conic equals the det-ratio of the undilated covariance, in [0, 1], 1 when
    culled -- the known answer of tests/test_antialiased.py:71-97, on the oracle's conics."""
    import splax_b200 as sx

    n, H, W = 3000, 128, 128
    m, s, q, c, op, bg = random_scene(n, 1)
    xys, d, r, cn, nth, cum = oracle_lib.project(m, s, np.roll(q, -1, -1), viewmat(), op, n=n,
                                                 **cam(H, W))
    rho = sx.opacity_compensation(torch.tensor(cn), torch.tensor(r)).numpy()
    eps = 0.3
    a, b, cc = cn[:, 0].astype(np.float64), cn[:, 1].astype(np.float64), cn[:, 2].astype(np.float64)
    live = r > 0
    det_conic = a * cc - b * b
    det_d = np.where(live, 1.0 / np.where(det_conic == 0, 1.0, det_conic), 1.0)
    cxx, cyy, cxy = cc * det_d, a * det_d, -b * det_d
    det_o = (cxx - eps) * (cyy - eps) - cxy * cxy
    ref = np.sqrt(np.clip(np.where(live, det_o / det_d, 1.0), 0.0, 1.0))
    assert np.allclose(rho[live], ref[live], atol=1e-5)
    assert np.all(rho >= 0.0) and np.all(rho <= 1.0)
    assert np.allclose(rho[~live], 1.0)
    assert rho[live].min() < 0.98


def test_look_at_convention():
    from splax_b200.utils import look_at

    vm = look_at(np.array([0.0, 0.0, 4.0]), np.zeros(3))
    p = vm[:3, :3] @ np.zeros(3) + vm[:3, 3]
    assert np.allclose(p, [0, 0, 4])  # the target sits on the optical axis at depth 4
    up = vm[:3, :3] @ np.array([0.0, 1.0, 0.0])
    assert up[1] < 0  # world up maps to image up (-y, OpenCV)
    assert np.allclose(vm[:3, :3] @ vm[:3, :3].T, np.eye(3), atol=1e-6)


def test_synthetic_scenes_are_seeded():
    from splax_b200.utils import synthetic_scene

    a = synthetic_scene(2, n=1000)
    b = synthetic_scene(2, n=1000)
    assert all(np.array_equal(a[k], b[k]) for k in ("means", "scales", "quats", "colors",
                                                     "opacities", "viewmats"))
    assert a["viewmats"].shape == (8, 4, 4) and a["H"] == 1080 and a["W"] == 1920


def test_nvls_allreduce_argument_checks(lib):
    """The gradient all-reduce refuses bad ranks, sizes, epochs and alignment before any launch."""
    import ctypes

    from splax_b200 import _lib

    flags = (ctypes.c_void_p * 2)(16, 32)
    err = ctypes.c_void_p(64)
    f = lib.splax_nvls_allreduce_f32
    ok = dict(mc=ctypes.c_void_p(1 << 20), rank=0, world=2, n=8, epoch=1)
    for bad in (dict(world=9), dict(world=0), dict(rank=2), dict(rank=-1), dict(n=-1),
                dict(epoch=0), dict(mc=ctypes.c_void_p((1 << 20) + 4)), dict(mc=None)):
        a = {**ok, **bad}
        rc = f(a["mc"], flags, a["rank"], a["world"], a["n"], ctypes.c_uint64(a["epoch"]), err,
               None)
        assert rc == _lib.SPLAX_ERR_INVALID_ARGUMENT, bad


def test_nvls_adam_argument_checks(lib):
    """The fused exchange-and-Adam step refuses bad groups, steps, ranks and epochs before any
    launch; the shard lengths of the ranks cover the buffer once."""
    import ctypes

    from splax_b200 import _lib

    flags = (ctypes.c_void_p * 2)(16, 32)
    sizes = (ctypes.c_int64 * 2)(6, 5)
    lrs = (ctypes.c_float * 2)(1e-3, 1e-2)
    P = ctypes.c_void_p
    ok = dict(n=11, groups=2, step=1, rank=0, world=2, epoch=1)
    for bad in (dict(n=12), dict(groups=0), dict(groups=9), dict(step=0), dict(rank=2),
                dict(world=9), dict(epoch=0)):
        a = {**ok, **bad}
        rc = lib.splax_nvls_adam_step(P(1 << 20), P(1 << 21), P(1 << 22), P(1 << 23), P(1 << 24),
                                      a["n"], a["groups"], sizes, lrs, a["step"], 0.9, 0.999,
                                      1e-8, flags, a["rank"], a["world"],
                                      ctypes.c_uint64(a["epoch"]), P(64), None)
        assert rc == _lib.SPLAX_ERR_INVALID_ARGUMENT, bad
    for n in (0, 3, 11, 1001, 9009):
        for world in (1, 2, 3, 8):
            total = 0
            for rank in range(world):
                ln = ctypes.c_int64(-1)
                assert lib.splax_nvls_adam_shard_len(n, rank, world, ctypes.byref(ln)) == 0
                total += ln.value
            assert total == n, (n, world)


def test_bench_reference_arm_contract():
    """`bench.py --impl reference` (the CPU arm the driver runs) prints one JSON line with the
    contract's keys, here on a small scene."""
    import json
    import subprocess
    import sys

    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--n", "2000"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e", "impl"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0
