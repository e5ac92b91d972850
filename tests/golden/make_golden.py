"""Generate tests/golden/*.npz: float64 numpy restatements of the reference formulas.

This is an independent second restatement of the splax projection (splax/_project/_kernels.py:
155-248), the ellipse tile count (splax/_intersect.py:47-183) and the forward blend
(splax/_rasterize/_kernels.py:124-205), written vectorised in float64 with numpy and sharing
no code with the C oracle. The C oracle (fp32) must agree with it to fp32 rounding, which
catches transcription errors in either. Run: python tests/golden/make_golden.py
"""

from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BW = 16


def quat_to_mat(q):  # xyzw
    x, y, z, w = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R = np.empty((q.shape[0], 3, 3))
    R[:, 0, 0] = 1 - 2 * (y * y + z * z)
    R[:, 0, 1] = 2 * (x * y - w * z)
    R[:, 0, 2] = 2 * (x * z + w * y)
    R[:, 1, 0] = 2 * (x * y + w * z)
    R[:, 1, 1] = 1 - 2 * (x * x + z * z)
    R[:, 1, 2] = 2 * (y * z - w * x)
    R[:, 2, 0] = 2 * (x * z - w * y)
    R[:, 2, 1] = 2 * (y * z + w * x)
    R[:, 2, 2] = 1 - 2 * (x * x + y * y)
    return R


def tile_count(A, B, C, t, px, py, tbx, tby):
    """Tiles a single ellipse touches: the AccuTile column walk in float64."""
    disc = B * B - A * C
    nt = -t / disc
    xe, ye = np.sqrt(nt * C), np.sqrt(nt * A)
    bmin, bmax = [px - xe, py - ye], [px + xe, py + ye]
    amin = [py + B * xe / C, px + B * ye / A]
    amax = [py - B * xe / C, px - B * ye / A]
    rmin = [max(0, min(tbx, int(bmin[0] / BW))), max(0, min(tby, int(bmin[1] / BW)))]
    rmax = [max(0, min(tbx, int(bmax[0] / BW + 1))), max(0, min(tby, int(bmax[1] / BW + 1)))]
    xs, ys = rmax[0] - rmin[0], rmax[1] - rmin[1]
    if xs * ys == 0:
        return 0
    isY = ys < xs
    if isY:
        rmin, rmax, bmin, bmax = rmin[::-1], rmax[::-1], bmin[::-1], bmax[::-1]
        amin, amax = amin[::-1], amax[::-1]
        pu, pv, coeff = py, px, A
    else:
        pu, pv, coeff = px, py, C

    def inter(coord):
        h = coord - pu
        sq = np.sqrt(disc * h * h + t * coeff)
        return ((-B * h - sq) / coeff + pv, (-B * h + sq) / coeff + pv)

    line0 = rmin[0] * BW
    Imin = inter(line0) if bmin[0] <= line0 else (bmax[1], bmin[1])
    count = 0
    for u in range(rmin[0], rmax[0]):
        lo, hi = u * BW, u * BW + BW
        Imax = inter(hi) if hi <= bmax[0] else Imin
        emin = bmin[1] if lo <= amin[1] < hi else min(Imin[0], Imax[0])
        emax = bmax[1] if lo <= amax[1] < hi else max(Imin[1], Imax[1])
        mn = max(rmin[1], min(rmax[1], int(emin / BW)))
        mx = min(rmax[1], max(rmin[1], int(emax / BW + 1)))
        count += mx - mn
        Imin = Imax
    return count


def project64(means, scales, quats_xyzw, vm, opac, H, W, fx, fy, cx, cy, clip=0.01):
    n = means.shape[0]
    Wr, tr = vm[:3, :3].astype(np.float64), vm[:3, 3].astype(np.float64)
    p = means.astype(np.float64) @ Wr.T + tr
    M = quat_to_mat(quats_xyzw.astype(np.float64)) * scales.astype(np.float64)[:, None, :]
    V = M @ np.transpose(M, (0, 2, 1))
    limx, limy = 1.3 * 0.5 * W / fx, 1.3 * 0.5 * H / fy
    tz = p[:, 2]
    tx = tz * np.clip(p[:, 0] / tz, -limx, limx)
    ty = tz * np.clip(p[:, 1] / tz, -limy, limy)
    J = np.zeros((n, 3, 3))
    J[:, 0, 0] = fx / tz
    J[:, 0, 2] = -fx * tx / tz**2
    J[:, 1, 1] = fy / tz
    J[:, 1, 2] = -fy * ty / tz**2
    T = J @ Wr
    cov = T @ V @ np.transpose(T, (0, 2, 1))
    cxx, cxy, cyy = cov[:, 0, 0] + 0.3, cov[:, 0, 1], cov[:, 1, 1] + 0.3
    det = cxx * cyy - cxy * cxy
    conic = np.stack([cyy / det, -cxy / det, cxx / det], -1)
    center = np.stack([p[:, 0] / (tz + 1e-6) * fx + cx, p[:, 1] / (tz + 1e-6) * fy + cy], -1)
    tbx, tby = (W + BW - 1) // BW, (H + BW - 1) // BW
    t = np.minimum(3.33**2, 2 * np.log(opac.astype(np.float64) * 255.0))
    rx, ry = np.ceil(np.sqrt(t * cxx)), np.ceil(np.sqrt(t * cyy))
    radii = np.zeros(n, np.int64)
    nth = np.zeros(n, np.int64)
    xys, depths, conics = np.zeros((n, 2)), np.zeros(n), np.zeros((n, 3))
    for i in range(n):
        if tz[i] <= clip or opac[i] < 1 / 255.0:
            continue
        if (center[i, 0] + rx[i] <= 0 or center[i, 0] - rx[i] >= W or center[i, 1] + ry[i] <= 0
                or center[i, 1] - ry[i] >= H):
            continue
        k = tile_count(*conic[i], t[i], *center[i], tbx, tby)
        if k <= 0:
            continue
        nth[i], depths[i], radii[i] = k, tz[i], int(max(rx[i], ry[i]))
        xys[i], conics[i] = center[i], conic[i]
    return xys, depths, radii, conics, nth


def blend64(colors, opac, bg, xys, depths, conics, radii, H, W):
    """Per-pixel front-to-back blend with a float64 sort by depth (all visible gaussians)."""
    vis = np.nonzero(radii > 0)[0]
    order = vis[np.argsort(depths[vis], kind="stable")]
    img = np.zeros((H, W, 3))
    T_final = np.ones((H, W))
    ys, xs = np.mgrid[0:H, 0:W] + 0.5
    T = np.ones((H, W))
    done = np.zeros((H, W), bool)
    acc = np.zeros((H, W, 3))
    for g in order:
        dx, dy = xys[g, 0] - xs, xys[g, 1] - ys
        a, b, c = conics[g]
        sigma = 0.5 * (a * dx * dx + c * dy * dy) + b * dx * dy
        alpha = np.minimum(0.999, opac[g] * np.exp(-sigma))
        ok = (~done) & (sigma >= 0) & (alpha >= 1 / 255.0)
        nT = T * (1 - alpha)
        stop = ok & (nT <= 1e-4)
        done |= stop
        ok &= ~stop
        acc += np.where(ok[..., None], colors[g] * (alpha * T)[..., None], 0.0)
        T = np.where(ok, nT, T)
    T_final = T
    img = acc + T_final[..., None] * bg
    return img, T_final


def main() -> None:
    rng = np.random.default_rng(20260)
    n, H, W = 600, 72, 88
    means = (rng.normal(size=(n, 3)) * 0.6).astype(np.float32)
    scales = rng.uniform(0.02, 0.1, size=(n, 3)).astype(np.float32)
    q = rng.normal(size=(n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    opac = rng.uniform(0.05, 0.95, size=n).astype(np.float32)
    bg = np.array([0.2, 0.5, 0.9], np.float32)
    vm = np.array([[1, 0, 0, 0.1], [0, 1, 0, -0.2], [0, 0, 1, 4.5], [0, 0, 0, 1]], np.float32)
    fx = fy = 80.0
    cx, cy = W / 2, H / 2
    xys, depths, radii, conics, nth = project64(means, scales, q, vm, opac, H, W, fx, fy, cx, cy)
    img, T = blend64(colors, opac, bg, xys, depths, conics, radii, H, W)
    np.savez_compressed(
        HERE / "projection_blend_f64.npz", means=means, scales=scales, quats_xyzw=q,
        colors=colors, opac=opac, bg=bg, viewmat=vm, img_shape=np.array([H, W]),
        f=np.array([fx, fy]), c=np.array([cx, cy]), xys=xys, depths=depths, radii=radii,
        conics=conics, nth=nth, img=img, final_T=T)
    print("wrote", HERE / "projection_blend_f64.npz", "visible", int((radii > 0).sum()),
          "tiles", int(nth.sum()))


if __name__ == "__main__":
    main()
