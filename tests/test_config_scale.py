"""GPU parity at the headline configuration's full size (config 2 of the benchmark).

N = 1,000,000 gaussians (means normal(0, 1.5)), 1080x1920 images, f = 1400, the ring cameras of
the benchmark (radius 5, height 1), the same seeded scene ``bench.py`` times:

- one camera, forward and backward: projection bit-exact, sorted ids, keys and bins bit-exact,
  the image within max-abs 1e-4 (and final_idx equal) on every pixel the oracle does not flag,
  the gradients of the five parameter arrays and the viewmat within relative L2 1e-3 (the image
  cotangent masked on flagged pixels, as in the smaller render test);
- all eight cameras at once: the batched projection bit-exact and the intersection sort on the
  64-bit key path the reference falls back to at B=8 (splax/_rasterize/_sort/_sort.py:51-66;
  tests/test_warp_rasterize.py:310-359) bit-exact, ~64M intersections.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4
GRAD_TOL = 1e-3


@pytest.fixture(scope="module")
def sx():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import splax_b200

    return splax_b200


@pytest.fixture(scope="module")
def scene():
    from splax_b200 import utils

    sc = utils.synthetic_scene(2)
    sc["cam"] = {"img_shape": (sc["H"], sc["W"]), "f": (sc["f"], sc["f"]),
                 "c": (sc["W"] / 2, sc["H"] / 2)}
    return sc


def T(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda")


def N(t):
    return t.detach().cpu().numpy()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30)


def _sort_cuda(xys, depths, radii, conics, map_opac, cum, n, B, H, W, key_bits):
    from splax_b200 import _lib

    lib = _lib.load()
    count = int(np.uint32(N(cum).reshape(-1)[-1]))
    Tn = ((W + 15) // 16) * ((H + 15) // 16)
    gids = torch.zeros(max(count, 1), dtype=torch.int32, device="cuda")
    keys = torch.zeros(max(count, 1), dtype=torch.int64, device="cuda")
    bins = torch.zeros((B * Tn, 2), dtype=torch.int32, device="cuda")
    ni, kb = ctypes.c_int64(0), ctypes.c_int32(0)
    p = _lib.ptr
    mo = map_opac.reshape(-1).contiguous()
    rc = lib.splax_sort_and_bin(p(xys), p(depths), p(radii), p(conics), p(mo), mo.numel(),
                                p(cum), n, B, H, W, key_bits, p(gids), gids.numel(), p(keys),
                                p(bins), ctypes.byref(ni), ctypes.byref(kb),
                                _lib.stream_of(xys))
    _lib.check(rc)
    _lib.check(lib.splax_check_device_errors(_lib.stream_of(xys)))
    return N(gids)[:count], N(keys)[:count], N(bins), ni.value, kb.value


def test_config2_camera_fwd_bwd_full_size(sx, oracle_lib, scene):
    import _oracle_chain as ch

    m, s, q, c, op = (scene[k] for k in ("means", "scales", "quats", "colors", "opacities"))
    bg = scene["background"]
    n, H, W = m.shape[0], scene["H"], scene["W"]
    vm = scene["viewmats"][0]
    kw = scene["cam"]
    # projection: every output bit-exact
    cu = sx.project(T(m), T(s), T(q), T(vm), opacities=T(op), **kw)
    orc = oracle_lib.project(m, s, np.roll(q, -1, -1), vm, op, n=n, **kw)
    for k, name in enumerate(["xys", "depths", "radii", "conics", "num_tiles_hit", "cum"]):
        a = N(cu[k]).reshape(orc[k].shape)
        assert np.array_equal(a, orc[k]), (name, int((a != orc[k]).sum()))
    xys, d, r, cn, nth, cum = cu
    # sort and bin: ids, keys and bins bit-exact
    g_c, k_c, b_c, count, kb_c = _sort_cuda(xys, d, r, cn, T(op), cum, n, 1, H, W, 0)
    rc, g_o, k_o, b_o, kb_o = oracle_lib.sort_and_bin(*orc[:4], op, orc[5], n=n, B=1,
                                                      img_shape=(H, W))
    assert rc == 0 and kb_c == kb_o == 32 and count == len(g_o) > 5_000_000
    assert np.array_equal(k_c, k_o)
    assert np.array_equal(g_c, g_o)
    assert np.array_equal(b_c, b_o)
    del g_c, k_c, b_c, g_o, k_o, b_o
    # forward image and residuals
    from splax_b200._rasterize import _RasterizeFn

    img, fT, fi = _RasterizeFn.apply(T(c), T(op), T(op), T(bg).reshape(1, 3), xys, d, r, cn,
                                     cum, n, H, W, 0, False, 0)
    fT_o, fi_o, img_o, _, flags = oracle_lib.rasterize(c, op, op, bg, *orc[:4], orc[5], n=n, B=1,
                                                       img_shape=(H, W))
    flags = flags.reshape(H, W)
    ok = flags == 0
    assert ok.mean() > 0.99, int((~ok).sum())
    assert np.abs(N(img).reshape(H, W, 3) - img_o.reshape(H, W, 3))[ok].max() <= IMG_TOL
    assert np.array_equal(N(fi).reshape(H, W)[ok], fi_o.reshape(H, W)[ok])
    # gradients of the five parameter arrays and the viewmat
    w = np.random.default_rng(7).uniform(size=(H, W, 3)).astype(np.float32) / (H * W)
    w[~ok] = 0.0
    params = [T(x).requires_grad_() for x in (m, s, q, c, op)]
    vm_t = T(vm).requires_grad_()
    img2, _ = sx.render(*params, viewmat=vm_t, background=T(bg), **kw)
    (img2 * T(w)).sum().backward()
    ref = ch.grads(m, s, q, c, op, bg, vm, w, **kw)
    names = ["means", "scales", "quats", "colors", "opacities"]
    errs = {nm: rel_l2(N(pt.grad), g) for nm, pt, g in zip(names, params, ref[:5])}
    errs["viewmat"] = rel_l2(N(vm_t.grad), ref[5])
    assert max(errs.values()) <= GRAD_TOL, errs


def test_config2_eight_camera_sort_64bit_full_size(sx, oracle_lib, scene):
    m, s, q, op = (scene[k] for k in ("means", "scales", "quats", "opacities"))
    n, H, W = m.shape[0], scene["H"], scene["W"]
    views = scene["viewmats"]
    B = views.shape[0]
    kw = scene["cam"]
    cu = sx.project(T(m), T(s), T(q), T(views), opacities=T(op), **kw)
    orc = oracle_lib.project(m, s, np.roll(q, -1, -1), views.reshape(-1, 4), op, n=n, B=B, **kw)
    for k, name in enumerate(["xys", "depths", "radii", "conics", "num_tiles_hit", "cum"]):
        a = N(cu[k]).reshape(orc[k].shape)
        assert np.array_equal(a, orc[k]), (name, int((a != orc[k]).sum()))
    xys, d, r, cn, nth, cum = cu
    g_c, k_c, b_c, count, kb_c = _sort_cuda(xys, d, r, cn, T(op), cum, n, B, H, W, 0)
    rc, g_o, k_o, b_o, kb_o = oracle_lib.sort_and_bin(*orc[:4], op, orc[5], n=n, B=B,
                                                      img_shape=(H, W))
    assert rc == 0 and kb_c == kb_o == 64 and count == len(g_o) > 50_000_000
    assert np.array_equal(g_c, g_o)
    assert np.array_equal(b_c, b_o)
    assert np.array_equal(k_c, k_o)
