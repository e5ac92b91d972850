"""GPU parity of the plain FFI-target backward entry points, called through the C ABI.

These are the symbols an XLA FFI binding of the reference's ``project_bwd``,
``rasterize_bwd`` and ``rasterize_bwd_depth`` targets would bind
(splax/_project/_kernels.py:344-353, splax/_rasterize/_kernels.py:503-512,917-926); the torch
layer uses the ``_ex`` variants, so these tests drive the plain ones with ctypes, in the
reference's argument order and batch conventions, against the C oracle:

- K14 (``_project_bwd_kernel``, splax/_project/_kernels.py:356-606) for one camera, a viewmat
  stack with per-image ``v_viewmat`` (tests/test_warp_grad_batched.py:170-188), batched means,
  and rigid ``gaussian_transforms`` shared by the batch or stacked per image with
  ``v_transforms`` (tests/test_transforms.py:357-421);
- the rasterize backward with broadcast geometry, B_geom = 1 < B_out, and an image cotangent
  arriving broadcast (H rows) or batched (B_out*H rows), background shared or per image
  (splax/_rasterize/_kernels.py:408-419,558-568,598-601; tests/test_warp_grad_batched.py:190-214).

Bar: relative L2 <= 1e-3 for every gradient array (per image for v_viewmat).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cam, random_scene, viewmat

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from splax_b200 import _lib

    return _lib.load()


def T(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda")


def N(t):
    return t.detach().cpu().numpy()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30)


def _rigid(rng, k):
    """k rigid 4x4 transforms: a rotation about a random axis plus a small shift."""
    out = np.zeros((k, 4, 4), np.float32)
    for i in range(k):
        ax = rng.normal(size=3)
        ax /= np.linalg.norm(ax)
        ang = rng.uniform(-0.4, 0.4)
        Kx = np.array([[0, -ax[2], ax[1]], [ax[2], 0, -ax[0]], [-ax[1], ax[0], 0]])
        R = np.eye(3) + np.sin(ang) * Kx + (1 - np.cos(ang)) * Kx @ Kx
        out[i, :3, :3] = R
        out[i, :3, 3] = rng.uniform(-0.2, 0.2, size=3)
        out[i, 3, 3] = 1.0
    return out


def _project_bwd_ffi(lib, m, s, q_xyzw, vm, radii, conics, vxy, vd, vc, tf, ids, n, K, has_tf,
                     f, B):
    from splax_b200 import _lib

    total = B * n
    outs = [torch.full((total, 3), 7.0, device="cuda"), torch.full((total, 3), 7.0, device="cuda"),
            torch.full((total, 4), 7.0, device="cuda"), torch.full((B, 4, 4), 7.0, device="cuda"),
            torch.full((B, K, 4, 4), 7.0, device="cuda")]
    p = _lib.ptr
    rc = lib.splax_project_bwd(
        p(m), m.numel() // 3, p(s), s.numel() // 3, p(q_xyzw), q_xyzw.numel() // 4, p(vm),
        vm.numel() // 4, p(radii), radii.numel(), p(conics), conics.numel() // 3, p(vxy),
        vxy.numel() // 2, p(vd), vd.numel(), p(vc), vc.numel() // 3, p(tf), tf.numel() // 16,
        p(ids), n, K, int(has_tf), f[0], f[1], 1.0, total, *[p(o) for o in outs],
        _lib.stream_of(m))
    _lib.check(rc)
    torch.cuda.synchronize()
    return [N(o) for o in outs]


CASES = {
    # name: (B, batched means, transforms: None | "shared" | "stacked")
    "single": (1, False, None),
    "viewmat_stack": (3, False, None),
    "batched_means": (3, True, None),
    "transforms_shared": (3, False, "shared"),
    "transforms_stacked": (2, False, "stacked"),
    "transforms_single": (1, False, "shared"),
}


@pytest.mark.parametrize("case", list(CASES))
def test_project_bwd_ffi_matches_oracle(lib, oracle_lib, case):
    B, batched_means, tf_mode = CASES[case]
    n, H, W = 6000, 192, 256
    m, s, q, c, op, bg = random_scene(n, 31, spread=0.8)
    rng = np.random.default_rng(32)
    q_xyzw = np.roll(q, -1, -1)
    views = (viewmat() if B == 1 else
             np.stack([viewmat(0.15 * i - 0.1, 0.05 * i, 4.5 + 0.3 * i) for i in range(B)]))
    vm_rows = views.reshape(-1, 4)
    means = m
    if batched_means:
        means = (m[None] + 0.05 * rng.normal(size=(B, n, 3))).astype(np.float32).reshape(B * n, 3)
    K = 2
    has_tf = tf_mode is not None
    if has_tf:
        base = _rigid(rng, K)
        tf = base if tf_mode == "shared" else np.stack(
            [_rigid(rng, K) for _ in range(B)]).reshape(B * K, 4, 4)
        ids = np.full(n, -1, np.int32)
        ids[: n // 3] = 0
        ids[n // 3: 2 * n // 3] = 1
    else:
        tf = np.zeros((1, 4, 4), np.float32)
        ids = np.full((1,), -1, np.int32)
    kw = dict(n=n, B=B, img_shape=(H, W), **{k: v for k, v in cam(H, W).items()
                                             if k != "img_shape"})
    tf_kw = dict(transforms=tf, transform_ids=ids, num_transforms=K) if has_tf else {}
    xys, d, r, cn, nth, cum = oracle_lib.project(means, s, q_xyzw, vm_rows, op, **kw, **tf_kw)
    assert (r > 0).sum() > 0.3 * B * n  # most pairs are visible
    vxy = rng.normal(size=(B * n, 2)).astype(np.float32)
    vd = rng.normal(size=(B * n,)).astype(np.float32)
    vc = rng.normal(size=(B * n, 3)).astype(np.float32)
    f = cam(H, W)["f"]
    got = _project_bwd_ffi(lib, T(means), T(s), T(q_xyzw), T(vm_rows), T(r, torch.int32), T(cn),
                           T(vxy), T(vd), T(vc), T(tf), T(ids, torch.int32), n, K if has_tf else 1,
                           has_tf, f, B)
    ref = oracle_lib.project_bwd(means, s, q_xyzw, vm_rows, r, cn, vxy, vd, vc, n=n, B=B, f=f,
                                 **tf_kw)
    names = ["v_mean3d", "v_scale", "v_quat", "v_viewmat", "v_transforms"]
    for name, a, b in zip(names[:3], got[:3], ref[:3]):
        e = rel_l2(a.reshape(b.shape), b)
        assert e <= GRAD_TOL, (case, name, e)
    for i in range(B):  # the camera pose gradient of every image
        e = rel_l2(got[3][i], ref[3][i])
        assert e <= GRAD_TOL, (case, "v_viewmat", i, e)
    if has_tf:
        gt = got[4].reshape(B, K, 4, 4)
        rt = ref[4].reshape(B, K, 4, 4)
        assert np.abs(rt).max() > 0
        for i in range(B):
            e = rel_l2(gt[i], rt[i])
            assert e <= GRAD_TOL, (case, "v_transforms", i, e)
    else:
        assert not got[4].any()  # overwritten with zeros


def _raster_fwd_ffi(lib, c, op, bg, xys, d, r, cn, cum, n, H, W, B):
    from splax_b200 import _lib

    fT = torch.empty((B * H, W), device="cuda")
    fi = torch.empty((B * H, W), device="cuda", dtype=torch.int32)
    img = torch.empty((B * H, W, 3), device="cuda")
    p = _lib.ptr
    _lib.check(lib.splax_rasterize(p(c), c.numel() // 3, p(op), op.numel(), p(op), op.numel(),
                                   p(bg), bg.numel() // 3, p(xys), p(d), p(r), p(cn), p(cum),
                                   B * n, n, H, W, B * H, 0, p(fT), p(fi), p(img),
                                   _lib.stream_of(c)))
    return fT, fi, img


@pytest.mark.parametrize("depth", [False, True])
@pytest.mark.parametrize("broadcast_cot,bg_rows", [(True, 1), (False, 1), (False, 3)])
def test_rasterize_bwd_ffi_broadcast_geometry(lib, oracle_lib, depth, broadcast_cot, bg_rows):
    """One render (B_geom = 1) differentiated against B_out = 3 target images: every output
    image gets its own gradient slot (grad_rows = 3n), read from the one geometry."""
    from splax_b200 import _lib

    n, H, W, B_out = 12_000, 160, 224, 3
    m, s, q, c, op, bg = random_scene(n, 41)
    xys, d, r, cn, nth, cum = oracle_lib.project(m, s, np.roll(q, -1, -1), viewmat(), op, n=n,
                                                 **cam(H, W))
    bgs = np.stack([bg, bg[::-1], 0.5 * bg]).astype(np.float32)[:bg_rows]
    t = dict(c=T(c), op=T(op), xys=T(xys), d=T(d), r=T(r, torch.int32), cn=T(cn),
             cum=T(cum, torch.int32))
    # the forward of the shared render (the background of image 0)
    bg0 = T(bgs[:1])
    fT, fi, img = _raster_fwd_ffi(lib, t["c"], t["op"], bg0, t["xys"], t["d"], t["r"], t["cn"],
                                  t["cum"], n, H, W, 1)
    rng = np.random.default_rng(42)
    rows = H if broadcast_cot else B_out * H
    v_img = rng.uniform(-1, 1, size=(rows, W, 3)).astype(np.float32)
    v_dep = rng.uniform(-1, 1, size=(rows, W)).astype(np.float32) if depth else None
    outs = [torch.full((B_out * n, 3), 9.0, device="cuda"), torch.full((B_out * n,), 9.0, device="cuda"),
            torch.full((B_out * n, 2), 9.0, device="cuda"), torch.full((B_out * n, 3), 9.0, device="cuda")]
    p = _lib.ptr
    bg_t, vimg_t = T(bgs), T(v_img)  # held until the kernels have run
    common = [p(t["c"]), n, p(t["op"]), n, p(t["op"]), n, p(bg_t), bg_rows, p(t["xys"]),
              p(t["d"]), p(t["r"]), p(t["cn"]), p(t["cum"]), n, p(fT), p(fi), p(vimg_t), rows]
    vd_t = T(v_dep) if depth else None
    if depth:
        outs.append(torch.full((B_out * n,), 9.0, device="cuda"))
        rc = lib.splax_rasterize_bwd_depth(*common, p(vd_t), rows, n, H, W, B_out * n, 0,
                                           *[p(o) for o in outs], _lib.stream_of(t["c"]))
    else:
        rc = lib.splax_rasterize_bwd(*common, n, H, W, B_out * n, 0, *[p(o) for o in outs],
                                     _lib.stream_of(t["c"]))
    _lib.check(rc)
    torch.cuda.synchronize()
    ref = oracle_lib.rasterize_bwd(c, op, op, bgs, xys, d, r, cn, cum, N(fT), N(fi), v_img,
                                   v_dep, n=n, B_out=B_out, B_geom=1, img_shape=(H, W))
    names = ["v_colors", "v_opacity", "v_xy", "v_conic", "v_depths"]
    for name, a, b in zip(names, [N(o) for o in outs], ref):
        if b is None:
            continue
        b = b.reshape(B_out, n, -1)
        a = a.reshape(b.shape)
        for i in range(B_out):  # each output image's slot
            e = rel_l2(a[i], b[i])
            assert e <= GRAD_TOL, (name, i, e)
    if broadcast_cot and bg_rows == 1:
        # identical cotangent rows and background: every image's slot is the same gradient
        a = N(outs[0]).reshape(B_out, n, 3)
        assert rel_l2(a[1], a[0]) <= 1e-5 and rel_l2(a[2], a[0]) <= 1e-5
