"""CPU checks of the C oracle itself, before it is trusted as the CUDA path's parity checker.

Ports of the reference's own known-answer tests and invariants (no GPU, no reference runtime):
- emit == count slot ownership and cum == cumsum (tests/test_warp_rasterize.py:433-487,
  tests/test_warp_batch.py:102-126)
- single-gaussian expected depth D == pvz * A (tests/test_depth_reg.py:75-107)
- key width choice and its fallback at B=8, 1080p (tests/test_warp_rasterize.py:310-359)
- packed vs 64-bit keys >= 65 dB (tests/test_warp_rasterize.py:264-289)
- batch invariance under the 64-bit key (tests/test_warp_batch.py:45-56, 129-244)
- finite-difference gradients (tests/test_warp_grad.py:147-184, 240-263)
plus agreement with the independent float64 restatement in tests/golden.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from conftest import cam, random_scene, viewmat

GOLDEN = Path(__file__).resolve().parent / "golden"


def _project(o, n, H, W, seed=0, vm=None, **kw):
    m, s, q, c, op, bg = random_scene(n, seed, **kw)
    vm = viewmat() if vm is None else vm
    out = o.project(m, s, np.roll(q, -1, -1), vm, op, n=n, **cam(H, W))
    return (m, s, q, c, op, bg, vm), out


def test_logf_matches_libm(oracle_lib):
    x = np.concatenate([np.geomspace(1e-38, 1e38, 4001), np.linspace(0.5, 2.0, 2001),
                        np.array([1.0, 255.0, 1 / 0.00392157])]).astype(np.float32)
    got = oracle_lib.logf(x).astype(np.float64)
    ref = np.log(x.astype(np.float64))
    ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    ulp = np.maximum(ulp, np.spacing(np.float32(1e-7)))
    assert np.all(np.abs(got - ref) <= 4 * ulp + 1e-7)


@pytest.mark.parametrize("n,H,W", [(20_000, 256, 256), (60_000, 512, 384)])
def test_emit_matches_count(oracle_lib, n, H, W):
    _, (xys, d, r, cn, nth, cum) = _project(oracle_lib, n, H, W, seed=n, spread=1.0,
                                            smin=0.005, smax=0.05, omin=0.0, omax=1.0)
    assert cum[-1] > 0
    np.testing.assert_array_equal(cum.astype(np.int64), np.cumsum(nth.astype(np.int64)))
    opac = random_scene(n, n, spread=1.0, smin=0.005, smax=0.05, omin=0.0, omax=1.0)[4]
    rc, keys, gids = oracle_lib.map_intersects(xys, d, r, cn, opac, cum, n=n, B=1,
                                               img_shape=(H, W), key_bits_request=64)
    assert rc == 0
    assert not (keys == -999).any() and (gids >= 0).all()
    starts = np.concatenate([[0], cum[:-1]])
    for i in np.nonzero(nth > 0)[0][:3000]:
        assert (gids[starts[i]:cum[i]] == i).all()


def test_bins_partition_sorted_range(oracle_lib):
    n, H, W = 8000, 200, 300
    (m, s, q, c, op, bg, vm), (xys, d, r, cn, nth, cum) = _project(oracle_lib, n, H, W, 3)
    for kb_req in (0, 64):
        rc, gids, keys, bins, kb = oracle_lib.sort_and_bin(xys, d, r, cn, op, cum, n=n, B=1,
                                                           img_shape=(H, W),
                                                           key_bits_request=kb_req)
        assert rc == 0 and kb == (32 if kb_req == 0 else 64)
        assert np.all(np.diff(keys) >= 0)
        nz = bins[bins[:, 1] > bins[:, 0]]
        assert nz[:, 0].min() == 0 and nz[:, 1].max() == cum[-1]
        assert (np.diff(nz[:, 0]) > 0).all() and np.array_equal(nz[1:, 0], nz[:-1, 1])
        # per-tile lists hold exactly the gaussians whose tile walk emitted that tile
        assert (np.bincount(gids, minlength=n) == nth).all()


def test_single_gaussian_depth(oracle_lib):
    """D == pvz * A for one gaussian, the known answer of tests/test_depth_reg.py:75-107."""
    import _oracle_chain as ch

    H = W = 64
    means = np.array([[0.1, -0.05, 0.0]], np.float32)
    scales = np.array([[0.12, 0.12, 0.12]], np.float32)
    quats = np.array([[1.0, 0.0, 0.0, 0.0]], np.float32)
    opac = np.array([0.9], np.float32)
    vm = np.array([[1, 0, 0, 0.0], [0, 1, 0, 0.0], [0, 0, 1, 4.0], [0, 0, 0, 1]], np.float32)
    pvz = float((vm[:3, :3] @ means[0] + vm[:3, 3])[2])
    black = np.zeros(3, np.float32)
    img, _, _ = ch.render(means, scales, quats, np.ones((1, 3), np.float32), opac, black, vm,
                          **cam(H, W))
    A = img[..., 0]
    _, depth, _ = ch.render(means, scales, quats, np.full((1, 3), 0.5, np.float32), opac, black,
                            vm, depth=True, **cam(H, W))
    assert np.allclose(depth, pvz * A, atol=1e-4)
    assert depth[0, 0] == 0.0 and A[0, 0] == 0.0
    assert depth.max() > 0.5 * pvz


def test_depth_path_image_identical(oracle_lib):
    """The depth blend's image is the plain image byte for byte (tests/test_depth_reg.py:110-117)."""
    import _oracle_chain as ch

    m, s, q, c, op, bg = random_scene(4000, 1)
    a, _, _ = ch.render(m, s, q, c, op, bg, viewmat(), **cam(128, 128))
    b, _, _ = ch.render(m, s, q, c, op, bg, viewmat(), depth=True, **cam(128, 128))
    assert np.array_equal(a, b)


def test_key_width_rule(oracle_lib):
    # B=1 at 1080p packs (13 tile bits, 18 depth bits); B=8 leaves 15 < 16 and falls back
    assert oracle_lib.key_bits(1, 1080, 1920) == (32, 13, 18)
    assert oracle_lib.key_bits(8, 1080, 1920)[0] == 64
    assert oracle_lib.key_bits(4, 1080, 1920)[0] == 32
    # image + tile bits above 32 overflow the 64-bit key (splax/_rasterize/_sort/_sort.py:61-66)
    assert oracle_lib.key_bits(1 << 20, 4096, 8192)[0] == -1


def test_packed_vs_64bit(oracle_lib):
    n, H, W = 30_000, 256, 256
    (m, s, q, c, op, bg, vm), (xys, d, r, cn, nth, cum) = _project(oracle_lib, n, H, W, 7)
    imgs = []
    for kb in (32, 64):
        _, _, img, _, _ = oracle_lib.rasterize(c, op, op, bg, xys, d, r, cn, cum, n=n, B=1,
                                               img_shape=(H, W), key_bits_request=kb)
        imgs.append(img)
    diff = np.abs(imgs[0] - imgs[1])
    mse = float(np.mean((imgs[0] - imgs[1]) ** 2))
    psnr = 99.0 if mse == 0 else -10 * np.log10(mse)
    assert diff.max() < 0.05 and psnr > 65


def test_batch_invariance_64bit(oracle_lib):
    """Batched projection + render == per-image results, bit for bit, under the 64-bit key."""
    n, H, W = 5000, 96, 128
    m, s, q, c, op, bg = random_scene(n, 2)
    views = np.stack([viewmat(0.0), viewmat(0.3), viewmat(-0.2)])
    B = 3
    xyzw = np.roll(q, -1, -1)
    bx = oracle_lib.project(m, s, xyzw, views.reshape(12, 4), op, n=n, B=B, **cam(H, W))
    for i in range(B):
        ref = oracle_lib.project(m, s, xyzw, views[i], op, n=n, **cam(H, W))
        for k in range(5):
            np.testing.assert_array_equal(bx[k][i * n:(i + 1) * n], ref[k])
    nth = bx[4].astype(np.int64)
    np.testing.assert_array_equal(bx[5].astype(np.int64), np.cumsum(nth))
    xys, d, r, cn, _, cum = bx
    _, _, img, _, _ = oracle_lib.rasterize(c, op, op, bg, xys, d, r, cn, cum, n=n, B=B,
                                           img_shape=(H, W), key_bits_request=64)
    for i in range(B):
        ref = oracle_lib.project(m, s, xyzw, views[i], op, n=n, **cam(H, W))
        _, _, ri, _, _ = oracle_lib.rasterize(c, op, op, bg, *ref[:4], ref[5], n=n, B=1,
                                              img_shape=(H, W), key_bits_request=64)
        np.testing.assert_array_equal(img[i * H:(i + 1) * H], ri)


def test_against_float64_restatement(oracle_lib):
    g = np.load(GOLDEN / "projection_blend_f64.npz")
    H, W = (int(v) for v in g["img_shape"])
    n = g["means"].shape[0]
    xys, d, r, cn, nth, cum = oracle_lib.project(g["means"], g["scales"], g["quats_xyzw"],
                                                 g["viewmat"], g["opac"], n=n, img_shape=(H, W),
                                                 f=tuple(g["f"]), c=tuple(g["c"]))
    live = (r > 0) & (g["radii"] > 0)
    assert (r > 0).sum() == (g["radii"] > 0).sum()
    assert np.abs(xys[live] - g["xys"][live]).max() < 1e-3
    assert np.abs(d[live] - g["depths"][live]).max() < 1e-5
    rel = np.abs(cn[live] - g["conics"][live]) / (np.abs(g["conics"][live]).max(1, keepdims=True))
    assert rel.max() < 1e-4
    assert np.mean(nth == g["nth"]) > 0.99 and np.mean(r == g["radii"]) > 0.99
    _, _, img, _, _ = oracle_lib.rasterize(g["colors"], g["opac"], g["opac"], g["bg"], xys, d, r,
                                           cn, cum, n=n, B=1, img_shape=(H, W),
                                           key_bits_request=64)
    err = np.abs(img.reshape(H, W, 3) - g["img"])
    assert np.quantile(err, 0.999) < 2e-3 and err.mean() < 1e-4


def _fd_check(oracle_lib, seed, which):
    import _oracle_chain as ch

    # scene sizes of tests/test_warp_grad.py:154 (params) and :246 (viewmat)
    n, H, W = (400, 80, 80) if which == "params" else (4000, 120, 120)
    m, s, q, c, op, bg = random_scene(n, seed)
    vm = viewmat()
    w = np.random.default_rng(seed + 1).uniform(size=(H, W, 3)).astype(np.float32)
    v_img = w / w.size

    def loss(args, v):
        img, _, _ = ch.render(*args, bg, v, **cam(H, W))
        return float(np.sum(v_img.astype(np.float64) * img))

    args = [m, s, q, c, op]
    g = ch.grads(*args, bg, vm, v_img, **cam(H, W))
    eps = 2e-3 if which == "params" else 1e-3
    if which == "params":
        dirs = [gi / (np.linalg.norm(gi) + 1e-12) for gi in g[:5]]
        analytic = sum(float(np.vdot(gi, di)) for gi, di in zip(g[:5], dirs))
        plus = [(a + eps * d).astype(np.float32) for a, d in zip(args, dirs)]
        minus = [(a - eps * d).astype(np.float32) for a, d in zip(args, dirs)]
        numeric = (loss(plus, vm) - loss(minus, vm)) / (2 * eps)
    else:
        gv = g[5]
        assert np.allclose(gv[3], 0.0)
        d = np.zeros((4, 4), np.float32)
        d[:3] = gv[:3] / (np.linalg.norm(gv[:3]) + 1e-12)
        analytic = float(np.vdot(gv, d))
        numeric = (loss(args, vm + eps * d) - loss(args, vm - eps * d)) / (2 * eps)
    rel = abs(analytic - numeric) / (abs(numeric) + 1e-12)
    assert rel < 8e-2, (analytic, numeric)


def test_finite_difference_params(oracle_lib):
    _fd_check(oracle_lib, 7, "params")


def test_finite_difference_viewmat(oracle_lib):
    _fd_check(oracle_lib, 11, "viewmat")


def test_finite_difference_depth(oracle_lib):
    """The depth cotangent path (tests/test_depth_reg.py:121-152): FD of sum(w * depth)."""
    import _oracle_chain as ch

    n, H, W = 300, 64, 64
    m, s, q, c, op, bg = random_scene(n, 5)
    vm = viewmat()
    wd = np.random.default_rng(3).uniform(size=(H, W)).astype(np.float32) / (H * W)

    def loss(mm):
        _, dep, _ = ch.render(mm, s, q, c, op, bg, vm, depth=True, **cam(H, W))
        return float(np.sum(wd.astype(np.float64) * dep))

    g = ch.grads(m, s, q, c, op, bg, vm, np.zeros((H, W, 3), np.float32), v_depth_img=wd,
                 **cam(H, W))[0]
    d = g / (np.linalg.norm(g) + 1e-12)
    eps = 2e-3
    numeric = (loss((m + eps * d).astype(np.float32)) - loss((m - eps * d).astype(np.float32)))
    numeric /= 2 * eps
    analytic = float(np.vdot(g, d))
    assert abs(analytic - numeric) / (abs(numeric) + 1e-12) < 8e-2


def test_transform_identity_and_shift(oracle_lib):
    """A rigid transform equals moving the means by hand (splax/_project/_kernels.py:627-644)."""
    n, H, W = 2000, 96, 96
    m, s, q, c, op, bg = random_scene(n, 9)
    xyzw = np.roll(q, -1, -1)
    ang = 0.3
    R = np.array([[np.cos(ang), -np.sin(ang), 0], [np.sin(ang), np.cos(ang), 0], [0, 0, 1]],
                 np.float32)
    tf = np.eye(4, dtype=np.float32)[None].repeat(2, 0)
    tf[1, :3, :3] = R
    tf[1, :3, 3] = [0.1, -0.2, 0.05]
    ids = np.full(n, -1, np.int32)
    ids[500:1500] = 1
    ids[:100] = 0
    a = oracle_lib.project(m, s, xyzw, viewmat(), op, n=n, transforms=tf, transform_ids=ids,
                           num_transforms=2, **cam(H, W))
    m2 = m.copy()
    m2[500:1500] = m[500:1500] @ R.T + tf[1, :3, 3]
    # rotated covariance: R_tf * R(q) == R(q') for q' = q_tf * q
    b = oracle_lib.project(m2, s, xyzw, viewmat(), op, n=n, **cam(H, W))
    same = np.r_[0:500, 1500:n]
    for k in range(5):
        np.testing.assert_array_equal(a[k][same], b[k][same])
    assert np.allclose(a[0][500:1500], b[0][500:1500], atol=1e-3)
