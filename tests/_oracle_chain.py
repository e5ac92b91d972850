"""Forward and backward render composed from the oracle's stages, for CPU-side checks.

Mirrors splax.render (splax/_render.py:29-115) without JAX: project -> [antialias] -> rasterize,
and the chain of the custom vjps (splax/_project/_project.py:404-443,
splax/_rasterize/_rasterize.py:191-231). With ``antialias_eps`` the blend opacities are
``opacities * rho`` with rho = ``opacity_compensation(conics, radii, eps)``
(splax/_project/_project.py:95-117) evaluated in fp32 in the reference's operation order, the
tile intersection stays on the raw opacities (splax/_render.py:103-107), and rho's vjp --
what JAX's autodiff of that formula gives -- is taken here in float64 and chained into the
conic and opacity cotangents before the projection backward.
"""

from __future__ import annotations

import numpy as np

import oracle


def compensation(conics, radii, eps):
    """rho and rho2 of opacity_compensation (splax/_project/_project.py:113-117) in fp32: the
    Python-float eps enters as float32(eps) and eps * eps as float32(eps * eps), no
    contraction, evaluated left to right as the reference writes it."""
    cn = np.asarray(conics, np.float32).reshape(-1, 3)
    a, b, c = cn[:, 0], cn[:, 1], cn[:, 2]
    e, e2 = np.float32(eps), np.float32(eps * eps)
    rho2 = (np.float32(1.0) - e * (a + c)) + e2 * (a * c - b * b)
    rho = np.sqrt(np.clip(rho2, np.float32(0.0), np.float32(1.0)))
    live = np.asarray(radii).reshape(-1) > 0
    return np.where(live, rho, np.float32(1.0)).astype(np.float32), rho2


def compensation_vjp(conics, radii, eps, v_rho):
    """Cotangent of the conics from rho's cotangent (float64): d rho / d rho2 = 1 / (2 rho)
    inside the clip, 0 where the clip is active or the pair is culled; d rho2 / d(a, b, c) =
    (-eps + eps^2 c, -2 eps^2 b, -eps + eps^2 a)."""
    cn = np.asarray(conics, np.float64).reshape(-1, 3)
    a, b, c = cn[:, 0], cn[:, 1], cn[:, 2]
    rho, rho2 = compensation(conics, radii, eps)
    inside = (np.asarray(radii).reshape(-1) > 0) & (rho2 > 0.0) & (rho2 < 1.0)
    v_rho2 = np.where(inside, np.asarray(v_rho, np.float64) / (2.0 * np.maximum(rho, 1e-30)), 0.0)
    return np.stack([v_rho2 * (-eps + eps * eps * c), v_rho2 * (-2.0 * eps * eps * b),
                     v_rho2 * (-eps + eps * eps * a)], axis=-1)


def render(means, scales, quats_wxyz, colors, opac, bg, vm, *, img_shape, f, c, depth=False,
           key_bits_request=0, antialias_eps=None):
    n = means.shape[0]
    xyzw = np.roll(quats_wxyz, -1, axis=-1)
    xys, d, r, cn, nth, cum = oracle.project(means, scales, xyzw, vm, opac, n=n,
                                             img_shape=img_shape, f=f, c=c)
    rho = None
    blend = opac
    if antialias_eps is not None:
        rho, _ = compensation(cn, r, antialias_eps)
        blend = (np.asarray(opac, np.float32).reshape(-1) * rho).astype(np.float32)
    fT, fi, img, dep, flags = oracle.rasterize(colors, blend, opac, bg, xys, d, r, cn, cum, n=n,
                                               B=1, img_shape=img_shape, with_depth=depth,
                                               key_bits_request=key_bits_request)
    H, W = img_shape
    state = dict(xys=xys, depths=d, radii=r, conics=cn, nth=nth, cum=cum, final_Ts=fT,
                 final_idx=fi, flags=flags, rho=rho, blend=blend)
    return img.reshape(H, W, 3), (None if dep is None else dep.reshape(H, W)), state


def grads(means, scales, quats_wxyz, colors, opac, bg, vm, v_img, *, img_shape, f, c,
          v_depth_img=None, antialias_eps=None):
    """Gradients of sum(v_img * render) (+ sum(v_depth_img * depth)) w.r.t. the five params
    (quats in wxyz) and the viewmat."""
    n = means.shape[0]
    H, W = img_shape
    img, dep, st = render(means, scales, quats_wxyz, colors, opac, bg, vm, img_shape=img_shape,
                          f=f, c=c, depth=v_depth_img is not None, antialias_eps=antialias_eps)
    vc, vo, vxy, vcon, vdep = oracle.rasterize_bwd(
        colors, st["blend"], opac, bg, st["xys"], st["depths"], st["radii"], st["conics"],
        st["cum"], st["final_Ts"], st["final_idx"], v_img.reshape(H, W, 3),
        None if v_depth_img is None else v_depth_img.reshape(H, W), n=n, B_out=1, B_geom=1,
        img_shape=img_shape)
    if antialias_eps is not None:
        # blend = opac * rho: the opacity takes v_blend * rho, rho takes v_blend * opac
        v_blend = np.asarray(vo, np.float64).reshape(-1)
        vo = (v_blend * st["rho"]).astype(np.float32)
        v_rho = v_blend * np.asarray(opac, np.float64).reshape(-1)
        v_cn = compensation_vjp(st["conics"], st["radii"], antialias_eps, v_rho)
        vcon = (np.asarray(vcon, np.float64).reshape(-1, 3) + v_cn).astype(np.float32)
    xyzw = np.roll(quats_wxyz, -1, axis=-1)
    v_depth = vdep if vdep is not None else np.zeros(n, np.float32)
    vm_, vs, vq, vv, _ = oracle.project_bwd(means, scales, xyzw, vm, st["radii"], st["conics"],
                                            vxy, v_depth, vcon, n=n, B=1, f=f)
    return vm_, vs, np.roll(vq, 1, axis=-1), vc, vo, vv[0]
