"""ctypes bindings of the C oracle (splat_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline / reference arm may
import this package. It is the parity checker for the CUDA path and never part of it.

Array arguments are numpy arrays in the reference's layouts (``splax/_project/_kernels.py:31-57``,
``splax/_rasterize/_kernels.py:37-54, 386-407``): per-gaussian rows of (N,3) / (N,4) / (N,) or,
batched, (B*N, ...); viewmats as (4,4) or (4B,4); images as (B*H, W[,3]).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "liboracle.so"
SOURCES = [_HERE / "splat_oracle.c"]
CFLAGS = ["-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC"]

_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle into oracle/liboracle.so with gcc (the checker, not the product)."""
    newest = max(p.stat().st_mtime for p in [*SOURCES, _HERE / "splat_oracle.h"])
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= newest:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["gcc", *CFLAGS, "-shared", "-o", str(tmp), *map(str, SOURCES), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
    return _lib


def _p(a: np.ndarray | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if a is None else a.ctypes.data)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _rows(a: np.ndarray, width: int) -> int:
    return a.size // width


I64, I32, F32, VP = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p


def logf(x: np.ndarray) -> np.ndarray:
    lib = _load()
    lib.orc_logf.restype = ctypes.c_float
    lib.orc_logf.argtypes = [ctypes.c_float]
    return np.array([lib.orc_logf(float(v)) for v in np.asarray(x, np.float32).ravel()], np.float32)


def key_bits(B: int, img_h: int, img_w: int, request: int = 0) -> tuple[int, int, int]:
    """(key_bits or -1 on overflow, tile_n_bits, depth_bits) per splax/_rasterize/_sort/_sort.py:51-66."""
    lib = _load()
    tnb, db = ctypes.c_int32(0), ctypes.c_int32(0)
    kb = lib.orc_key_bits(I32(B), I32(img_h), I32(img_w), ctypes.c_int(request),
                          ctypes.byref(tnb), ctypes.byref(db))
    return kb, tnb.value, db.value


def project(means3d, scales, quats_xyzw, viewmat, opacities, *, n: int, img_shape, f, c,
            glob_scale: float = 1.0, clip_thresh: float = 0.01, B: int = 1,
            transforms=None, transform_ids=None, num_transforms: int = 1, nthreads: int = 0):
    """K1 + K2. Returns xys (BN,2), depths (BN,), radii (BN,), conics (BN,3), nth (BN,), cum (BN,)."""
    lib = _load()
    m, s, q, vm, o = _f32(means3d), _f32(scales), _f32(quats_xyzw), _f32(viewmat), _f32(opacities)
    has_tf = transforms is not None
    tf = _f32(transforms) if has_tf else np.zeros((1, 4, 4), np.float32)
    ids = _i32(transform_ids) if has_tf else np.full((1,), -1, np.int32)
    K = tf.size // 16 if not has_tf else num_transforms
    total = B * n
    xys = np.zeros((total, 2), np.float32)
    depths = np.zeros(total, np.float32)
    radii = np.zeros(total, np.int32)
    conics = np.zeros((total, 3), np.float32)
    nth = np.zeros(total, np.int32)
    cum = np.zeros(total, np.int32)
    H, W = img_shape
    lib.orc_project(
        _p(m), I64(_rows(m, 3)), _p(s), I64(_rows(s, 3)), _p(q), I64(_rows(q, 4)), _p(vm),
        I64(_rows(vm, 4)), _p(o), I64(o.size), _p(tf), I64(tf.size // 16), _p(ids), I32(n),
        I32(K), I32(int(has_tf)), I32(H), I32(W), F32(f[0]), F32(f[1]), F32(c[0]), F32(c[1]),
        F32(glob_scale), F32(clip_thresh), I64(total), _p(xys), _p(depths), _p(radii),
        _p(conics), _p(nth), _p(cum), ctypes.c_int(nthreads))
    return xys, depths, radii, conics, nth, cum


def map_intersects(xys, depths, radii, conics, map_opacities, cum, *, n: int, B: int, img_shape,
                   key_bits_request: int = 0):
    """K5 only: keys and gaussian ids at the cum offsets, unsorted."""
    lib = _load()
    xys, depths, radii, conics = _f32(xys), _f32(depths), _i32(radii), _f32(conics)
    mo, cum = _f32(map_opacities), _i32(cum)
    count = int(np.uint32(cum[-1])) if cum.size else 0
    keys = np.full(max(count, 1), -999, np.int64)
    gids = np.full(max(count, 1), -1, np.int32)
    H, W = img_shape
    rc = lib.orc_map_intersects(_p(xys), _p(depths), _p(radii), _p(conics), _p(mo), I64(mo.size),
                                _p(cum), I32(n), I32(B), I32(H), I32(W),
                                ctypes.c_int(key_bits_request), _p(keys), _p(gids))
    return rc, keys[:count], gids[:count]


def sort_and_bin(xys, depths, radii, conics, map_opacities, cum, *, n: int, B: int, img_shape,
                 key_bits_request: int = 0):
    """sort_and_bin: (rc, gaussian_ids (I,), keys (I,) int64, tile_bins (B*T,2), key_bits)."""
    lib = _load()
    xys, depths, radii, conics = _f32(xys), _f32(depths), _i32(radii), _f32(conics)
    mo, cum = _f32(map_opacities), _i32(cum)
    count = int(np.uint32(cum[-1])) if cum.size else 0
    H, W = img_shape
    T = ((W + 15) // 16) * ((H + 15) // 16)
    gids = np.zeros(max(count, 1), np.int32)
    keys = np.zeros(max(count, 1), np.int64)
    bins = np.zeros((B * T, 2), np.int32)
    kb = ctypes.c_int32(0)
    rc = lib.orc_sort_and_bin(_p(xys), _p(depths), _p(radii), _p(conics), _p(mo), I64(mo.size),
                              _p(cum), I32(n), I32(B), I32(H), I32(W),
                              ctypes.c_int(key_bits_request), _p(gids), _p(keys), _p(bins),
                              ctypes.byref(kb), ctypes.c_int(0))
    return rc, gids[:count], keys[:count], bins, kb.value


def rasterize(colors, opacities, map_opacities, background, xys, depths, radii, conics, cum, *,
              n: int, B: int, img_shape, key_bits_request: int = 0, with_depth: bool = False,
              nthreads: int = 0):
    """K8 / K9: (final_Ts (B*H,W), final_idx (B*H,W), out_img (B*H,W,3), out_depth|None, flags)."""
    lib = _load()
    col, op, mo, bg = _f32(colors), _f32(opacities), _f32(map_opacities), _f32(background)
    xys, depths, radii, conics, cum = _f32(xys), _f32(depths), _i32(radii), _f32(conics), _i32(cum)
    H, W = img_shape
    fT = np.zeros((B * H, W), np.float32)
    fi = np.zeros((B * H, W), np.int32)
    img = np.zeros((B * H, W, 3), np.float32)
    dep = np.zeros((B * H, W), np.float32) if with_depth else None
    flags = np.zeros((B * H, W), np.uint8)
    rc = lib.orc_rasterize(_p(col), I64(_rows(col, 3)), _p(op), I64(op.size), _p(mo), I64(mo.size),
                           _p(bg), I64(_rows(bg, 3)), _p(xys), _p(depths), _p(radii), _p(conics),
                           _p(cum), I32(n), I32(B), I32(H), I32(W), ctypes.c_int(key_bits_request),
                           _p(fT), _p(fi), _p(img), _p(dep), _p(flags), ctypes.c_int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle rasterize failed with status {rc}")
    return fT, fi, img, dep, flags


def rasterize_bwd(colors, opacities, map_opacities, background, xys, depths, radii, conics, cum,
                  final_Ts, final_idx, v_out_img, v_out_depth=None, *, n: int, B_out: int,
                  B_geom: int, img_shape, key_bits_request: int = 0, nthreads: int = 0):
    """K10-K13: (v_colors, v_opacity, v_xy, v_conic, v_depths|None), each with B_out*n rows."""
    lib = _load()
    col, op, mo, bg = _f32(colors), _f32(opacities), _f32(map_opacities), _f32(background)
    xys, depths, radii, conics, cum = _f32(xys), _f32(depths), _i32(radii), _f32(conics), _i32(cum)
    fT, fi, vo = _f32(final_Ts), _i32(final_idx), _f32(v_out_img)
    H, W = img_shape
    vd = _f32(v_out_depth) if v_out_depth is not None else None
    rows = B_out * n
    v_colors = np.zeros((rows, 3), np.float32)
    v_opac = np.zeros(rows, np.float32)
    v_xy = np.zeros((rows, 2), np.float32)
    v_conic = np.zeros((rows, 3), np.float32)
    v_depths = np.zeros(rows, np.float32) if vd is not None else None
    rc = lib.orc_rasterize_bwd(
        _p(col), I64(_rows(col, 3)), _p(op), I64(op.size), _p(mo), I64(mo.size), _p(bg),
        I64(_rows(bg, 3)), _p(xys), _p(depths), _p(radii), _p(conics), _p(cum), _p(fT), _p(fi),
        _p(vo), I64(vo.size // (3 * W)), _p(vd), I64(0 if vd is None else vd.size // W), I32(n),
        I32(B_out), I32(B_geom), I32(H), I32(W), ctypes.c_int(key_bits_request), _p(v_colors),
        _p(v_opac), _p(v_xy), _p(v_conic), _p(v_depths), ctypes.c_int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle rasterize_bwd failed with status {rc}")
    return v_colors, v_opac, v_xy, v_conic, v_depths


def project_bwd(means3d, scales, quats_xyzw, viewmat, radii, conics, v_xy, v_depth, v_conic, *,
                n: int, B: int, f, glob_scale: float = 1.0, transforms=None, transform_ids=None,
                num_transforms: int = 1, nthreads: int = 0):
    """K14: (v_mean3d (BN,3), v_scale (BN,3), v_quat xyzw (BN,4), v_viewmat (B,4,4), v_transforms (B,K,4,4))."""
    lib = _load()
    m, s, q, vm = _f32(means3d), _f32(scales), _f32(quats_xyzw), _f32(viewmat)
    r, cn, vxy, vd, vc = _i32(radii), _f32(conics), _f32(v_xy), _f32(v_depth), _f32(v_conic)
    has_tf = transforms is not None
    tf = _f32(transforms) if has_tf else np.zeros((1, 4, 4), np.float32)
    ids = _i32(transform_ids) if has_tf else np.full((1,), -1, np.int32)
    K = num_transforms if has_tf else 1
    total = B * n
    v_mean = np.zeros((total, 3), np.float32)
    v_scale = np.zeros((total, 3), np.float32)
    v_quat = np.zeros((total, 4), np.float32)
    v_view = np.zeros((B, 4, 4), np.float32)
    v_tf = np.zeros((B, K, 4, 4), np.float32)
    lib.orc_project_bwd(
        _p(m), I64(_rows(m, 3)), _p(s), I64(_rows(s, 3)), _p(q), I64(_rows(q, 4)), _p(vm),
        I64(_rows(vm, 4)), _p(r), I64(r.size), _p(cn), I64(_rows(cn, 3)), _p(vxy),
        I64(_rows(vxy, 2)), _p(vd), I64(vd.size), _p(vc), I64(_rows(vc, 3)), _p(tf),
        I64(tf.size // 16), _p(ids), I32(n), I32(K), I32(int(has_tf)), F32(f[0]), F32(f[1]),
        F32(glob_scale), I32(B), _p(v_mean), _p(v_scale), _p(v_quat), _p(v_view), _p(v_tf),
        ctypes.c_int(nthreads))
    return v_mean, v_scale, v_quat, v_view, v_tf


def tile_counts(xys, radii, conics, map_opacities, *, img_shape) -> np.ndarray:
    """Ellipse-walk tile count per gaussian for the given screen-space geometry."""
    lib = _load()
    xys, radii, conics, mo = _f32(xys), _i32(radii), _f32(conics), _f32(map_opacities)
    out = np.zeros(radii.size, np.int32)
    H, W = img_shape
    lib.orc_tile_counts(_p(xys), _p(radii), _p(conics), _p(mo), I64(mo.size), I64(radii.size),
                        I32(H), I32(W), _p(out))
    return out


def counters() -> dict:
    lib = _load()
    out = (ctypes.c_int64 * 5)()
    lib.orc_counters(out)
    keys = ["intersections", "fwd_evals", "fwd_contribs", "bwd_evals", "bwd_contribs"]
    return dict(zip(keys, list(out)))
