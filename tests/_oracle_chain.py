"""Forward and backward render composed from the oracle's stages, for CPU-side checks.

Mirrors splax.render (splax/_render.py:29-115) without JAX: project -> [antialias] -> rasterize,
and the chain of the custom vjps (splax/_project/_project.py:404-443,
splax/_rasterize/_rasterize.py:191-231).
"""

from __future__ import annotations

import numpy as np

import oracle


def render(means, scales, quats_wxyz, colors, opac, bg, vm, *, img_shape, f, c, depth=False,
           key_bits_request=0):
    n = means.shape[0]
    xyzw = np.roll(quats_wxyz, -1, axis=-1)
    xys, d, r, cn, nth, cum = oracle.project(means, scales, xyzw, vm, opac, n=n,
                                             img_shape=img_shape, f=f, c=c)
    fT, fi, img, dep, flags = oracle.rasterize(colors, opac, opac, bg, xys, d, r, cn, cum, n=n,
                                               B=1, img_shape=img_shape, with_depth=depth,
                                               key_bits_request=key_bits_request)
    H, W = img_shape
    state = dict(xys=xys, depths=d, radii=r, conics=cn, nth=nth, cum=cum, final_Ts=fT,
                 final_idx=fi, flags=flags)
    return img.reshape(H, W, 3), (None if dep is None else dep.reshape(H, W)), state


def grads(means, scales, quats_wxyz, colors, opac, bg, vm, v_img, *, img_shape, f, c,
          v_depth_img=None):
    """Gradients of sum(v_img * render) (+ sum(v_depth_img * depth)) w.r.t. the five params
    (quats in wxyz) and the viewmat."""
    n = means.shape[0]
    H, W = img_shape
    img, dep, st = render(means, scales, quats_wxyz, colors, opac, bg, vm, img_shape=img_shape,
                          f=f, c=c, depth=v_depth_img is not None)
    vc, vo, vxy, vcon, vdep = oracle.rasterize_bwd(
        colors, opac, opac, bg, st["xys"], st["depths"], st["radii"], st["conics"], st["cum"],
        st["final_Ts"], st["final_idx"], v_img.reshape(H, W, 3),
        None if v_depth_img is None else v_depth_img.reshape(H, W), n=n, B_out=1, B_geom=1,
        img_shape=img_shape)
    xyzw = np.roll(quats_wxyz, -1, axis=-1)
    v_depth = vdep if vdep is not None else np.zeros(n, np.float32)
    vm_, vs, vq, vv, _ = oracle.project_bwd(means, scales, xyzw, vm, st["radii"], st["conics"],
                                            vxy, v_depth, vcon, n=n, B=1, f=f)
    return vm_, vs, np.roll(vq, 1, axis=-1), vc, vo, vv[0]
