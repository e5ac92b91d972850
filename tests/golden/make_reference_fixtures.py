"""Generate tests/golden/reference_kernels.npz by running the reference's own kernel source.

The reference's hot-path kernels are Warp-DSL Python (splax/_project/_kernels.py,
splax/_intersect.py, splax/_rasterize/_sort/_kernels.py) driven by plain host code
(splax/_rasterize/_sort/_sort.py). warp-lang is not installable here, so ``warp_standin``
supplies Warp's Python API on the CPU and this script executes, unmodified:

- ``_project_warp`` (splax/_project/_kernels.py:31-107): the batch selectors, the launch of
  ``_project_kernel`` (:122-248, with _apply_transform / _project_geom / _load_affine and the
  ellipse walk of splax/_intersect.py:47-183) and the inclusive scan;
- ``sort_and_bin`` (splax/_rasterize/_sort/_sort.py:29-171): the key-width rule, the depth
  range kernels (splax/_rasterize/_sort/_kernels.py:31-73), the key emission of 32- or 64-bit
  keys (:76-211), the stable sort and the bin edges (:214-269);

on small seeded scenes that exercise the paths the reference's tests exercise: one and several
cameras, 32-bit and forced 64-bit keys (the ``_use_32bit_keys`` hook,
tests/test_warp_rasterize.py:310-359), rigid transforms shared or stacked per image, large
footprints walked along either axis, gaussians behind the camera, off screen or below the
alpha threshold, and ragged image sizes.

Each case stores its inputs and the reference code's outputs. ``tests/test_reference_fixtures.py``
compares the C oracle (CPU) and the CUDA path (GPU) with them bit for bit. The script also
reports how many tile counts change when ``wp.log`` is the C library's float32 log instead of
the atanh-series log both implementations evaluate (the stored fixtures use the latter).

Run (needs the reference source tree, a few minutes of CPU):
    python tests/golden/make_reference_fixtures.py /path/to/reference
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import warp_standin as wp  # noqa: E402

OUT = HERE / "reference_kernels.npz"


def look(dx, dy, dz):
    return np.array([[1, 0, 0, dx], [0, 1, 0, dy], [0, 0, 1, dz], [0, 0, 0, 1]], np.float32)


def rotz(a, dz):
    c, s = np.cos(a), np.sin(a)
    return np.array([[c, -s, 0, 0.1], [s, c, 0, -0.05], [0, 0, 1, dz], [0, 0, 0, 1]], np.float32)


def rigid(rng, k):
    out = np.zeros((k, 4, 4), np.float32)
    for i in range(k):
        ax = rng.normal(size=3)
        ax /= np.linalg.norm(ax)
        ang = rng.uniform(-0.5, 0.5)
        K = np.array([[0, -ax[2], ax[1]], [ax[2], 0, -ax[0]], [-ax[1], ax[0], 0]])
        out[i, :3, :3] = np.eye(3) + np.sin(ang) * K + (1 - np.cos(ang)) * K @ K
        out[i, :3, 3] = rng.uniform(-0.3, 0.3, size=3)
        out[i, 3, 3] = 1.0
    return out


def scene(rng, n, spread, smin, smax, omin=0.0, omax=1.0):
    means = (rng.normal(size=(n, 3)) * spread).astype(np.float32)
    scales = rng.uniform(smin, smax, size=(n, 3)).astype(np.float32)
    q = rng.normal(size=(n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    opac = rng.uniform(omin, omax, size=n).astype(np.float32)
    return means, scales, q, opac  # q is stored xyzw, as the Warp kernels take it


def cases():
    rng = np.random.default_rng(2024)
    out = {}
    m, s, q, o = scene(rng, 3000, 0.6, 0.005, 0.08)
    out["single"] = dict(means=m, scales=s, quats=q, opac=o, views=look(0.2, -0.1, 4.0)[None],
                         H=200, W=256, f=(220.0, 220.0), c=(128.0, 100.0), key64=False,
                         bwd=True)
    m, s, q, o = scene(rng, 1000, 0.6, 0.005, 0.06)
    views = np.stack([look(0.0, 0.0, 4.0), rotz(0.3, 4.5), look(-0.3, 0.2, 3.5)])
    out["batched32"] = dict(means=m, scales=s, quats=q, opac=o, views=views, H=96, W=144,
                            f=(120.0, 120.0), c=(72.0, 48.0), key64=False, bwd=True)
    out["batched64"] = dict(out["batched32"], key64=True, bwd=False)
    m, s, q, o = scene(rng, 250, 0.8, 0.1, 0.6, 0.05, 1.0)
    out["large"] = dict(means=m, scales=s, quats=q, opac=o, views=look(0.1, 0.05, 5.0)[None],
                        H=256, W=320, f=(260.0, 260.0), c=(160.0, 128.0), key64=False)
    m, s, q, o = scene(rng, 600, 0.5, 0.01, 0.08)
    ids = np.full(600, -1, np.int32)
    ids[:200] = 0
    ids[200:450] = 1
    out["transforms_shared"] = dict(means=m, scales=s, quats=q, opac=o,
                                    views=np.stack([look(0.0, 0.0, 4.0), rotz(-0.2, 4.2)]),
                                    H=96, W=128, f=(110.0, 110.0), c=(64.0, 48.0), key64=False,
                                    tf=rigid(rng, 2), ids=ids, bwd=True)
    out["transforms_stacked"] = dict(out["transforms_shared"],
                                     tf=np.concatenate([rigid(rng, 2), rigid(rng, 2)]))
    m, s, q, o = scene(rng, 800, 3.0, 0.002, 0.2, 0.0, 1.0)
    m[:20, 2] = -6.0  # behind the camera
    o[20:40] = rng.uniform(0.0, 1.0 / 255.0, size=20).astype(np.float32)  # below threshold
    out["edge"] = dict(means=m, scales=s, quats=q, opac=o, views=look(0.0, 0.0, 4.0)[None],
                       H=37, W=91, f=(60.0, 60.0), c=(45.5, 18.5), key64=False, bwd=True)
    m, s, q, o = scene(rng, 300, 0.7, 0.01, 0.1)
    views = np.stack([rotz(0.25 * k - 0.5, 3.8 + 0.2 * k) for k in range(5)])
    out["five_cameras"] = dict(means=m, scales=s, quats=q, opac=o, views=views, H=40, W=72,
                               f=(50.0, 50.0), c=(36.0, 20.0), key64=False)
    # exactly one intersection: the bin-edge kernel's early return at index 0 leaves end = 0
    m = np.array([[0.01, 0.02, 0.0], [0.0, 0.0, -9.0], [0.3, 0.1, -9.0]], np.float32)
    s = np.full((3, 3), 0.004, np.float32)
    q = np.tile(np.array([[0, 0, 0, 1]], np.float32), (3, 1))
    o = np.array([0.5, 0.5, 0.5], np.float32)
    out["one_intersection"] = dict(means=m, scales=s, quats=q, opac=o,
                                   views=look(0.0, 0.0, 4.0)[None], H=64, W=64, f=(60.0, 60.0),
                                   c=(40.0, 40.0), key64=False)
    out["no_intersection"] = dict(out["one_intersection"], means=m + np.float32([0, 0, -9]))
    # blends: forward (K8 / K9) and backward (K10 staged or K11 warp-aggregated, by the
    # reference's own launch gate), for seeded colours, backgrounds and image cotangents
    m, s, q, o = scene(rng, 600, 0.5, 0.01, 0.07, 0.1, 1.0)
    out["blend_single"] = dict(means=m, scales=s, quats=q, opac=o, views=look(0.1, 0.0, 4.0)[None],
                               H=64, W=96, f=(90.0, 90.0), c=(48.0, 32.0), key64=False,
                               blend=dict(depth=False, B_out=1, cot_rows=64, bg_rows=1))
    m, s, q, o = scene(rng, 400, 0.5, 0.01, 0.07, 0.1, 1.0)
    out["blend_depth_batched"] = dict(
        means=m, scales=s, quats=q, opac=o, views=np.stack([look(0.0, 0.0, 4.0), rotz(0.2, 4.3)]),
        H=48, W=64, f=(70.0, 70.0), c=(32.0, 24.0), key64=False,
        blend=dict(depth=True, B_out=2, cot_rows=96, bg_rows=2))
    m, s, q, o = scene(rng, 2500, 0.35, 0.03, 0.12, 0.05, 0.6)
    out["blend_dense"] = dict(means=m, scales=s, quats=q, opac=o, views=look(0.0, 0.0, 4.0)[None],
                              H=48, W=48, f=(80.0, 80.0), c=(24.0, 24.0), key64=False,
                              blend=dict(depth=False, B_out=1, cot_rows=48, bg_rows=1))
    m, s, q, o = scene(rng, 300, 0.5, 0.01, 0.07, 0.1, 1.0)
    out["blend_broadcast"] = dict(means=m, scales=s, quats=q, opac=o,
                                  views=look(0.0, 0.1, 4.0)[None], H=40, W=56, f=(60.0, 60.0),
                                  c=(28.0, 20.0), key64=False,
                                  blend=dict(depth=True, B_out=2, cot_rows=40, bg_rows=1))
    return out


def run_blend(mods, cs, n, B, H, W, geom):
    """_rasterize(_depth)_warp and _rasterize_bwd(_depth)_warp (splax/_rasterize/_kernels.py:
    37-87, 208-262, 386-500, 797-914) on the projected geometry of the case."""
    bl = cs["blend"]
    rng = np.random.default_rng(int(n) * 7 + B)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    bg = rng.uniform(size=(bl["bg_rows"], 3)).astype(np.float32)
    v_img = rng.uniform(-1, 1, size=(bl["cot_rows"], W, 3)).astype(np.float32)
    v_dep = rng.uniform(-1, 1, size=(bl["cot_rows"], W)).astype(np.float32)
    xys, depths, radii, conics, cum = geom
    rk = mods["raster_kernels"]
    res = dict(colors=colors, bg=bg, cot_img=v_img,
               final_Ts=np.zeros((B * H, W), np.float32), final_idx=np.zeros((B * H, W), np.int32),
               out_img=np.zeros((B * H, W, 3), np.float32))
    fwd_in = [arr(colors, wp.vec3), arr(cs["opac"], wp.float32), arr(cs["opac"], wp.float32),
              arr(bg, wp.vec3), xys, depths, radii, conics, cum, n, H, W]
    fT, fi = arr(res["final_Ts"], wp.float32), arr(res["final_idx"], wp.int32)
    img = arr(res["out_img"], wp.vec3)
    if bl["depth"]:
        res["out_depth"] = np.zeros((B * H, W), np.float32)
        rk._rasterize_depth_warp(*fwd_in, fT, fi, img, arr(res["out_depth"], wp.float32))
    else:
        rk._rasterize_warp(*fwd_in, fT, fi, img)
    rows = bl["B_out"] * n
    for k, w in (("v_colors", 3), ("v_opacity", 0), ("v_xy", 2), ("v_conic", 3)):
        res[k] = np.zeros((rows, w) if w else rows, np.float32)
    grads = [arr(res["v_colors"], wp.vec3), arr(res["v_opacity"], wp.float32),
             arr(res["v_xy"], wp.vec2), arr(res["v_conic"], wp.vec3)]
    bwd_in = [arr(colors, wp.vec3), arr(cs["opac"], wp.float32), arr(cs["opac"], wp.float32),
              arr(bg, wp.vec3), xys, depths, radii, conics, cum, fT, fi, arr(v_img, wp.vec3)]
    if bl["depth"]:
        res["cot_depth"] = v_dep
        res["v_depths"] = np.zeros(rows, np.float32)
        rk._rasterize_bwd_depth_warp(*bwd_in, arr(v_dep, wp.float32), n, H, W, *grads,
                                     arr(res["v_depths"], wp.float32))
    else:
        rk._rasterize_bwd_warp(*bwd_in, n, H, W, *grads)
    return res


def arr(a, dt):
    return wp.array(np.ascontiguousarray(a), dt)


def run_case(mods, cs, log_kind="atanh"):
    wp.set_log(log_kind)
    n = cs["means"].shape[0]
    views = cs["views"]
    B = views.shape[0]
    total = B * n
    H, W = cs["H"], cs["W"]
    has_tf = "tf" in cs
    tf = cs["tf"] if has_tf else np.zeros((1, 4, 4), np.float32)
    ids = cs["ids"] if has_tf else np.full((1,), -1, np.int32)
    K = 2 if has_tf else 1
    outs = dict(xys=np.zeros((total, 2), np.float32), depths=np.zeros(total, np.float32),
                radii=np.zeros(total, np.int32), conics=np.zeros((total, 3), np.float32),
                nth=np.zeros(total, np.int32), cum=np.zeros(total, np.int32))
    xys, depths = arr(outs["xys"], wp.vec2), arr(outs["depths"], wp.float32)
    radii, conics = arr(outs["radii"], wp.int32), arr(outs["conics"], wp.vec3)
    nth, cum = arr(outs["nth"], wp.int32), arr(outs["cum"], wp.int32)
    mods["project_kernels"]._project_warp(
        arr(cs["means"], wp.vec3), arr(cs["scales"], wp.vec3), arr(cs["quats"], wp.quat),
        arr(views.reshape(-1, 4), wp.float32), arr(cs["opac"], wp.float32),
        arr(tf, wp.float32), arr(ids, wp.int32), n, K, has_tf, H, W, cs["f"][0], cs["f"][1],
        cs["c"][0], cs["c"][1], 1.0, 0.01, xys, depths, radii, conics, nth, cum)
    srt = mods["sort"]
    srt._use_32bit_keys = (lambda depth_bits: False) if cs["key64"] else \
        (lambda depth_bits: depth_bits >= 16)
    sys.modules["splax._cache"].state.clear()
    gids, bins, count, tbx, ntiles = srt.sort_and_bin(
        xys, depths, radii, conics, arr(cs["opac"], wp.float32), cum, n, B, H, W)
    if cs.get("bwd", False):
        # projection backward: _project_bwd_warp (splax/_project/_kernels.py:257-341) with its
        # tiled kernel (:356-484) and vjps (:487-606), for seeded cotangents of every pair
        rng = np.random.default_rng(int(total))
        v_xy = rng.normal(size=(total, 2)).astype(np.float32)
        v_depth = rng.normal(size=total).astype(np.float32)
        v_conic = rng.normal(size=(total, 3)).astype(np.float32)
        grads = dict(v_mean3d=np.zeros((total, 3), np.float32),
                     v_scale=np.zeros((total, 3), np.float32),
                     v_quat=np.zeros((total, 4), np.float32),
                     v_viewmat=np.zeros((4 * B, 4), np.float32),
                     v_transforms=np.zeros((B * K, 4, 4), np.float32))
        mods["project_kernels"]._project_bwd_warp(
            arr(cs["means"], wp.vec3), arr(cs["scales"], wp.vec3), arr(cs["quats"], wp.quat),
            arr(views.reshape(-1, 4), wp.float32), radii, conics, arr(v_xy, wp.vec2),
            arr(v_depth, wp.float32), arr(v_conic, wp.vec3), arr(tf, wp.float32),
            arr(ids, wp.int32), n, K, has_tf, cs["f"][0], cs["f"][1], 1.0,
            arr(grads["v_mean3d"], wp.vec3), arr(grads["v_scale"], wp.vec3),
            arr(grads["v_quat"], wp.vec4), arr(grads["v_viewmat"], wp.float32),
            arr(grads["v_transforms"], wp.float32))
        outs.update(cot_v_xy=v_xy, cot_v_depth=v_depth, cot_v_conic=v_conic, **grads)
    sorted_keys = sys.modules["splax._cache"].state["isect_ids"].data
    outs.update(gaussian_ids=gids.data[:count].copy(),
                isect_ids=sorted_keys[:count].astype(np.int64), tile_bins=bins.data.copy(),
                count=np.int64(count), key_bits=np.int32(8 * sorted_keys.itemsize))
    if cs.get("blend"):
        ntiles = ((W + 15) // 16) * ((H + 15) // 16)
        outs["bwd_staged"] = np.bool_(count >= B * ntiles * 256)  # the reference's launch gate
        outs.update({"blend_" + k: v for k, v in
                     run_blend(mods, cs, n, B, H, W, (xys, depths, radii, conics, cum)).items()})
    return outs



def main(ref_root: str) -> None:
    mods = wp.load_reference(Path(ref_root))
    data, report = {}, {}
    for name, cs in cases().items():
        t0 = time.time()
        res = run_case(mods, cs)
        alt = run_case(mods, dict(cs, bwd=False, blend=None), "libm")
        report[name] = {
            "pairs": int(res["radii"].size), "visible": int((res["radii"] > 0).sum()),
            "intersections": int(res["count"]),
            "key_bits": int(res["key_bits"]),
            "libm_log_tile_counts_differ": int((alt["nth"] != res["nth"]).sum()),
            "seconds": round(time.time() - t0, 1)}
        print(name, report[name], flush=True)
        for k in ("means", "scales", "quats", "opac", "views", "H", "W", "f", "c", "key64"):
            data[f"{name}/{k}"] = np.asarray(cs[k])
        data[f"{name}/bwd"] = np.asarray(bool(cs.get("bwd", False)))
        if "tf" in cs:
            data[f"{name}/tf"] = cs["tf"]
            data[f"{name}/ids"] = cs["ids"]
        for k, v in res.items():
            data[f"{name}/out_{k}"] = np.asarray(v)
    np.savez_compressed(OUT, **data)
    (HERE / "reference_kernels.json").write_text(json.dumps(report, indent=1) + "\n")
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_reference_fixtures.py <reference source tree>")
    main(sys.argv[1])
