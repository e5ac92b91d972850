"""GPU parity of the CUDA path against the C oracle, through the C ABI and the torch API.

Bars (stated per test): integer stages (tile counts, radii, cum, keys, sorted ids, bins,
final_idx) bit-exact; projection floats bit-exact (same IEEE op order, no FMA); images
max-abs <= 1e-4 on every pixel whose threshold decisions the oracle does not flag as within
rounding distance (flagged pixels must stay under 1%); gradients relative L2 <= 1e-3.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import cam, random_scene, viewmat

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4
GRAD_TOL = 1e-3


@pytest.fixture(scope="module")
def sx():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import splax_b200

    return splax_b200


def T(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda")


def N(t):
    return t.detach().cpu().numpy()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30)


def _proj_both(sx, oracle_lib, n, H, W, seed, views=None, **scene_kw):
    m, s, q, c, op, bg = random_scene(n, seed, **scene_kw)
    views = viewmat() if views is None else views
    B = 1 if views.ndim == 2 else views.shape[0]
    out_cuda = sx.project(T(m), T(s), T(q), T(views), opacities=T(op), **cam(H, W))
    out_orc = oracle_lib.project(m, s, np.roll(q, -1, -1), views.reshape(-1, 4), op, n=n, B=B,
                                 **cam(H, W))
    return (m, s, q, c, op, bg, views, B), out_cuda, out_orc


@pytest.mark.parametrize("n,H,W,seed", [(20_000, 256, 256, 0), (50_000, 480, 640, 1),
                                        (7, 33, 47, 2), (3000, 17, 300, 3)])
def test_project_bit_exact(sx, oracle_lib, n, H, W, seed):
    _, cu, orc = _proj_both(sx, oracle_lib, n, H, W, seed, spread=1.0, smin=0.005, smax=0.05,
                            omin=0.0, omax=1.0)
    names = ["xys", "depths", "radii", "conics", "num_tiles_hit", "cum_tiles_hit"]
    for k, name in enumerate(names):
        a = N(cu[k]).reshape(orc[k].shape)
        assert np.array_equal(a, orc[k]), (name, int((a != orc[k]).sum()))


def test_large_gaussians_count_and_emission_bit_exact(sx, oracle_lib):
    """Gaussians spanning up to ~45 tile rows: the warp-cooperative walks (row chunks of 32 per
    warp, several chunks per warp) reproduce the sequential walk's counts and tiles."""
    n, H, W = 3000, 720, 1280
    scene, cu, orc = _proj_both(sx, oracle_lib, n, H, W, 11, spread=1.0, smin=0.05, smax=0.6,
                                omin=0.0, omax=1.0)
    for k in range(6):
        a = N(cu[k]).reshape(orc[k].shape)
        assert np.array_equal(a, orc[k]), k
    nth = N(cu[4]).reshape(-1)
    assert nth.max() > 200  # large footprints are present
    xys, d, r, cn, _, cum = cu
    op = scene[4]
    g_c, k_c, b_c, count, _ = _sort_cuda(sx, xys, d, r, cn, T(op), cum, n, 1, H, W, 0)
    rc, g_o, k_o, b_o, _ = oracle_lib.sort_and_bin(*orc[:4], op, orc[5], n=n, B=1,
                                                   img_shape=(H, W))
    assert rc == 0 and count == len(g_o)
    assert np.array_equal(g_c, g_o)
    assert np.array_equal(b_c, b_o)


def test_project_batched_bit_exact(sx, oracle_lib):
    views = np.stack([viewmat(0.0), viewmat(0.3), viewmat(-0.2, 0.1, 4.0)])
    (_, _, _, _, _, _, _, B), cu, orc = _proj_both(sx, oracle_lib, 8000, 128, 160, 4, views)
    assert cu[0].shape == (3, 8000, 2)
    for k in range(6):
        assert np.array_equal(N(cu[k]).reshape(orc[k].shape), orc[k]), k
    nth = N(cu[4]).reshape(-1).astype(np.int64)
    assert np.array_equal(N(cu[5]).reshape(-1).astype(np.int64), np.cumsum(nth))


def _sort_cuda(sx, xys, depths, radii, conics, map_opac, cum, n, B, H, W, key_bits):
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


@pytest.mark.parametrize("key_bits", [0, 32, 64])
@pytest.mark.parametrize("n,H,W,B", [(30_000, 256, 256, 1), (20_000, 200, 330, 3),
                                     # 17-bit bin keys and 17/26-bit pair keys: 9-bit digits
                                     (6_000, 2160, 3840, 4)])
def test_sort_and_bin_bit_exact(sx, oracle_lib, key_bits, n, H, W, B):
    views = viewmat() if B == 1 else np.stack([viewmat(0.1 * i) for i in range(B)])
    (m, s, q, c, op, bg, _, _), cu, orc = _proj_both(sx, oracle_lib, n, H, W, 5, views)
    xys, d, r, cn, nth, cum = cu
    g_c, k_c, b_c, count, kb_c = _sort_cuda(sx, xys, d, r, cn, T(op), cum, n, B, H, W, key_bits)
    rc, g_o, k_o, b_o, kb_o = oracle_lib.sort_and_bin(*orc[:4], op, orc[5], n=n, B=B,
                                                      img_shape=(H, W),
                                                      key_bits_request=key_bits)
    assert rc == 0 and kb_c == kb_o and count == len(g_o)
    assert np.array_equal(k_c, k_o)
    assert np.array_equal(g_c, g_o)
    assert np.array_equal(b_c, b_o)


def _raster_inputs(sx, oracle_lib, n, H, W, seed, views=None):
    (m, s, q, c, op, bg, views, B), cu, orc = _proj_both(sx, oracle_lib, n, H, W, seed, views)
    return (m, s, q, c, op, bg, views, B), cu, orc


def _compare_images(img_c, img_o, flags, fi_c=None, fi_o=None):
    ok = flags == 0
    assert ok.mean() > 0.99, f"{(~ok).sum()} flagged pixels"
    d = np.abs(img_c - img_o)
    assert d[ok].max() <= IMG_TOL, d[ok].max()
    if fi_c is not None:
        assert np.array_equal(fi_c[ok], fi_o[ok])


@pytest.mark.parametrize("n,H,W,seed", [(4000, 128, 128, 1), (60_000, 320, 480, 2),
                                        (500, 37, 91, 3)])
def test_rasterize_parity(sx, oracle_lib, n, H, W, seed):
    (m, s, q, c, op, bg, views, B), cu, orc = _raster_inputs(sx, oracle_lib, n, H, W, seed)
    xys, d, r, cn, nth, cum = cu
    img = sx.rasterize(T(c), T(op), T(bg), xys, d, r, cn, cum, img_shape=(H, W))
    fT, fi, img_o, _, flags = oracle_lib.rasterize(c, op, op, bg, *orc[:4], orc[5], n=n, B=1,
                                                   img_shape=(H, W))
    _compare_images(N(img).reshape(H, W, 3), img_o.reshape(H, W, 3), flags.reshape(H, W))


def test_rasterize_zero_and_negative_blend_opacities(sx, oracle_lib):
    """Blend opacities that are zero or negative while the tile intersection uses positive map
    opacities (the rasterize API takes both): the reference skips such gaussians (alpha below
    1/255), and so must the blends, whose exponent carries log2 of the blend opacity."""
    n, H, W = 4000, 128, 160
    (m, s, q, c, op, bg, views, B), cu, orc = _raster_inputs(sx, oracle_lib, n, H, W, 9)
    xys, d, r, cn, nth, cum = cu
    blend = op.copy()
    rng = np.random.default_rng(19)
    pick = rng.permutation(n)
    blend[pick[: n // 8]] = 0.0
    neg = pick[n // 8: n // 4]
    blend[neg] = -rng.uniform(0.05, 0.9, size=neg.size).astype(np.float32)
    img = sx.rasterize(T(c), T(blend), T(bg), xys, d, r, cn, cum, img_shape=(H, W),
                       map_opacities=T(op))
    fT, fi, img_o, _, flags = oracle_lib.rasterize(c, blend, op, bg, *orc[:4], orc[5], n=n, B=1,
                                                   img_shape=(H, W))
    assert np.isfinite(N(img)).all()
    _compare_images(N(img).reshape(H, W, 3), img_o.reshape(H, W, 3), flags.reshape(H, W))


def test_rasterize_residuals_and_depth(sx, oracle_lib):
    from splax_b200._rasterize import _RasterizeFn

    n, H, W = 20_000, 200, 264
    (m, s, q, c, op, bg, views, B), cu, orc = _raster_inputs(sx, oracle_lib, n, H, W, 6)
    xys, d, r, cn, nth, cum = cu
    img, dep, fT, fi = _RasterizeFn.apply(T(c), T(op), T(op), T(bg).reshape(1, 3), xys, d, r,
                                          cn, cum, n, H, W, 0, True, 32)
    fT_o, fi_o, img_o, dep_o, flags = oracle_lib.rasterize(c, op, op, bg, *orc[:4], orc[5], n=n,
                                                           B=1, img_shape=(H, W),
                                                           with_depth=True)
    flags = flags.reshape(H, W)
    _compare_images(N(img), img_o.reshape(H, W, 3), flags, N(fi), fi_o)
    ok = flags == 0
    assert np.abs(N(fT) - fT_o)[ok].max() <= 1e-5
    assert np.abs(N(dep) - dep_o)[ok].max() <= 1e-3 * max(1.0, np.abs(dep_o).max())
    # the depth blend's image equals the plain image byte for byte (tests/test_depth_reg.py:110)
    img2 = sx.rasterize(T(c), T(op), T(bg), xys, d, r, cn, cum, img_shape=(H, W))
    assert torch.equal(img2, img)


def test_rasterize_bwd_parity(sx, oracle_lib):
    """Backward blend against the oracle fed the CUDA forward's residuals."""
    from splax_b200._rasterize import _RasterizeFn

    n, H, W = 30_000, 256, 320
    (m, s, q, c, op, bg, views, B), cu, orc = _raster_inputs(sx, oracle_lib, n, H, W, 7)
    xys, d, r, cn, nth, cum = cu
    cols, opac = T(c).requires_grad_(), T(op).requires_grad_()
    xy_t, cn_t, d_t = xys.clone().requires_grad_(), cn.clone().requires_grad_(), d.clone().requires_grad_()
    img, dep, fT, fi = _RasterizeFn.apply(cols, opac, T(op), T(bg).reshape(1, 3), xy_t, d_t, r,
                                          cn_t, cum, n, H, W, 0, True, 32)
    w = np.random.default_rng(9).uniform(size=(H, W, 3)).astype(np.float32)
    wd = np.random.default_rng(10).uniform(size=(H, W)).astype(np.float32)
    loss = (img * T(w)).sum() + (dep * T(wd)).sum()
    loss.backward()
    vc, vo, vxy, vcon, vdep = oracle_lib.rasterize_bwd(
        c, op, op, bg, *orc[:4], orc[5], N(fT), N(fi), w, wd, n=n, B_out=1, B_geom=1,
        img_shape=(H, W))
    for name, a, b in [("colors", cols.grad, vc), ("opacity", opac.grad, vo),
                       ("xy", xy_t.grad, vxy), ("conic", cn_t.grad, vcon), ("depth", d_t.grad, vdep)]:
        assert rel_l2(N(a).reshape(b.shape), b) <= GRAD_TOL, name


def _masked_cotangent(ch, m, s, q, c, op, bg, vm, H, W, seed):
    """A seeded image cotangent, zero on the pixels whose threshold decisions (alpha vs 1/255,
    T vs 1e-4, sigma's sign) the oracle flags as within rounding distance of the boundary: there
    the two implementations may legitimately take different branches, as in the image test."""
    _, _, st = ch.render(m, s, q, c, op, bg, vm, **cam(H, W))
    flags = st["flags"].reshape(H, W)
    assert (flags == 0).mean() > 0.99
    w = np.random.default_rng(seed).uniform(size=(H, W, 3)).astype(np.float32) / (H * W)
    w[flags != 0] = 0.0
    return w


def test_render_grads_vs_oracle(sx, oracle_lib):
    """End to end: torch autograd through render vs the oracle's vjp chain, the image cotangent
    masked on flagged pixels."""
    import _oracle_chain as ch

    n, H, W = 3000, 128, 128
    m, s, q, c, op, bg = random_scene(n, 11)
    vm = viewmat()
    w = _masked_cotangent(ch, m, s, q, c, op, bg, vm, H, W, 3)
    params = [T(x).requires_grad_() for x in (m, s, q, c, op)]
    vm_t = T(vm).requires_grad_()
    img, _ = sx.render(*params, viewmat=vm_t, background=T(bg), **cam(H, W))
    (img * T(w)).sum().backward()
    ref = ch.grads(m, s, q, c, op, bg, vm, w, **cam(H, W))
    names = ["means", "scales", "quats", "colors", "opacities"]
    errs = {name: rel_l2(N(pt.grad), g) for name, pt, g in zip(names, params, ref[:5])}
    errs["viewmat"] = rel_l2(N(vm_t.grad), ref[5])
    assert max(errs.values()) <= GRAD_TOL, errs


def test_batched_render_equals_stack_64bit(sx, monkeypatch):
    """Batch-native render == stack of single renders, bit for bit, under 64-bit keys
    (tests/test_warp_batch.py:45-56, 129-140)."""
    import splax_b200._sort as srt

    monkeypatch.setattr(srt, "_use_32bit_keys", lambda depth_bits: False)
    n, H, W = 8000, 128, 128
    m, s, q, c, op, bg = random_scene(n, 2)
    views = np.stack([viewmat(0.0), viewmat(0.3), viewmat(-0.2)])
    kw = dict(background=T(np.zeros(3)), **cam(H, W))
    out, _ = sx.render(T(m), T(s), T(q), T(c), T(op), viewmat=T(views), **kw)
    ref = torch.stack([sx.render(T(m), T(s), T(q), T(c), T(op), viewmat=T(v), **kw)[0]
                       for v in views])
    assert out.shape == ref.shape and torch.equal(out, ref)


def test_batched_grads_match_sequential(sx):
    n, H, W, B = 500, 96, 96, 3
    m, s, q, c, op, bg = random_scene(n, 2)
    bm = m[None] + 0.02 * np.random.default_rng(1).normal(size=(B, n, 3)).astype(np.float32)
    kw = dict(viewmat=T(viewmat()), background=T(bg), **cam(H, W))

    def grad_of(means):
        mt = T(means).requires_grad_()
        img, _ = sx.render(mt, T(s), T(q), T(c), T(op), **kw)
        img.sum().backward()
        return N(mt.grad)

    bt = T(bm).requires_grad_()
    img, _ = sx.render(bt, T(s), T(q), T(c), T(op), **kw)
    img.sum().backward()
    seq = np.stack([grad_of(bm[i]) for i in range(B)])
    for i in range(B):  # each image's means gradient (only the atomics' order differs)
        assert rel_l2(N(bt.grad)[i], seq[i]) <= GRAD_TOL, i


def test_key_width_fallback_and_overflow(sx):
    n, H, W = 4000, 1080, 1920
    m, s, q, c, op, bg = random_scene(n, 1)
    kw = dict(background=T(np.zeros(3)), **cam(H, W))
    sx.clear_cache()
    sx.render(T(m), T(s), T(q), T(c), T(op), viewmat=T(viewmat()), **kw)
    assert sx.scratch_info()["isect_dtype"] == torch.int32
    sx.clear_cache()
    views = np.stack([viewmat(dz=5.0 + 0.1 * i) for i in range(8)])
    sx.render(T(m), T(s), T(q), T(c), T(op), viewmat=T(views), **kw)
    assert sx.scratch_info()["isect_dtype"] == torch.int64
    sx.clear_cache()
    assert sx.scratch_info()["sig"] is None


def test_all_culled_and_tiny_batches(sx, oracle_lib):
    """No visible gaussian: the image is the background, the gradients are zero and no device
    error is raised. Then 5 gaussians seen by 5 cameras at an odd size match the oracle."""
    from splax_b200 import _lib

    n, H, W = 64, 37, 53
    m, s, q, c, op, bg = random_scene(n, 21)
    m = m.copy()
    m[:, 2] = -20.0  # behind every camera below
    params = [T(x).requires_grad_() for x in (m, s, q, c, op)]
    img, _ = sx.render(*params, viewmat=T(viewmat()), background=T(bg), **cam(H, W))
    assert torch.equal(img, T(bg).expand(H, W, 3))
    img.sum().backward()
    for p in params:
        assert p.grad is None or not bool(p.grad.any())
    _lib.check(_lib.load().splax_check_device_errors(_lib.stream_of(img)))

    n, B = 5, 5
    views = np.stack([viewmat(0.1 * i, 0.05 * i, 3.0 + 0.2 * i) for i in range(B)])
    (m, s, q, c, op, bg, views, B), cu, orc = _raster_inputs(sx, oracle_lib, n, H, W, 22, views)
    xys, d, r, cn, nth, cum = cu
    assert np.array_equal(N(nth).reshape(-1), orc[4])
    img = sx.rasterize(T(c), T(op), T(bg), xys, d, r, cn, cum, img_shape=(H, W))
    fT, fi, img_o, _, flags = oracle_lib.rasterize(c, op, op, bg, *orc[:4], orc[5], n=n, B=B,
                                                   img_shape=(H, W))
    _compare_images(N(img).reshape(B * H, W, 3), img_o.reshape(B * H, W, 3),
                    flags.reshape(B * H, W))


def test_scratch_reuse_across_sizes(sx):
    """A warm, differently sized scratch gives the same image as a cleared one
    (tests/test_warp_rasterize.py:211-228)."""
    for n, H, W in [(60_000, 300, 400), (10_000, 256, 256), (40_000, 512, 512), (10_000, 256, 256)]:
        m, s, q, c, op, bg = random_scene(n, n, spread=1.0, smin=0.005, smax=0.05)
        args = (T(m), T(s), T(q), T(c), T(op))
        kw = dict(viewmat=T(viewmat()), background=T(bg), **cam(H, W))
        warm, _ = sx.render(*args, **kw)
        sx.clear_cache()
        cold, _ = sx.render(*args, **kw)
        assert torch.equal(warm, cold)


def test_inconsistent_cum_is_reported(sx):
    """Geometry that disagrees with cum_tiles_hit raises instead of corrupting memory."""
    from splax_b200 import _lib

    n, H, W = 2000, 128, 128
    m, s, q, c, op, bg = random_scene(n, 3)
    xys, d, r, cn, nth, cum = sx.project(T(m), T(s), T(q), T(viewmat()), opacities=T(op),
                                         **cam(H, W))
    bad_cum = (cum - 1).clamp_min(0)
    bad_cum[-1] = cum[-1]
    with pytest.raises(_lib.SplaxDeviceError):
        sx.rasterize(T(c), T(op), T(bg), xys, d, r, cn, bad_cum, img_shape=(H, W))
        _lib.check(_lib.load().splax_check_device_errors(_lib.stream_of(xys)))
    # the error word is cleared and the next call works
    sx.rasterize(T(c), T(op), T(bg), xys, d, r, cn, cum, img_shape=(H, W))
    _lib.check(_lib.load().splax_check_device_errors(_lib.stream_of(xys)))


def test_key_overflow_raises(sx):
    import splax_b200._sort as srt

    with pytest.raises(ValueError, match="key overflow"):
        srt.key_bits_for(1 << 20, 4096, 8192)


def test_backward_reuses_forward_sort(sx):
    """The backward skips its re-sort when the forward's sort is still the device's latest one,
    and re-sorts (same gradients) when another render ran in between."""
    from splax_b200 import _lib

    n, H, W = 20_000, 200, 240
    m, s, q, c, op, bg = random_scene(n, 12)
    w = T(np.random.default_rng(5).uniform(size=(H, W, 3)))
    other = random_scene(5000, 13)

    def grads(intervene):
        params = [T(x).requires_grad_() for x in (m, s, q, c, op)]
        img, _ = sx.render(*params, viewmat=T(viewmat()), background=T(bg), **cam(H, W))
        if intervene:
            sx.render(*(T(x) for x in other[:5]), viewmat=T(viewmat()), background=T(bg),
                      **cam(H, W))
        (img * w).sum().backward()
        return [N(p.grad) for p in params]

    _lib.profile_reset()
    g_reuse = grads(False)
    reused = _lib.profile_report()["units"]["sort_reuses"]
    _lib.profile_reset()
    g_fresh = grads(True)
    fresh = _lib.profile_report()["units"]["sort_reuses"]
    assert reused == 1 and fresh == 0
    for a, b in zip(g_reuse, g_fresh):
        assert rel_l2(a, b) <= 1e-5
