"""Differentiable rasterization stage (splax/_rasterize/_rasterize.py), backed by libsplax_b200.

``rasterize`` / ``rasterize_depth`` keep the reference's signatures. The custom vjps become
``torch.autograd.Function``s whose residuals are the inputs plus the per-pixel final
transmittance and last contributing index. The backward re-runs the deterministic sort, so
the saved final_idx lines up exactly as in the reference (splax/_rasterize/_kernels.py:522-525).
"""

from __future__ import annotations

import torch

from splax_b200 import _lib, _sort


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.detach().to(torch.float32).contiguous()


def _i32(x: torch.Tensor) -> torch.Tensor:
    return x.detach().to(torch.int32).contiguous()


class _RasterizeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, colors, opacities, map_opacities, background, xys, depths, radii, conics,
                cum_tiles_hit, n, img_h, img_w, B, with_depth, key_bits):
        dev = _lib.require_cuda(colors, opacities, xys, conics)
        lib = _lib.load()
        col, op, mo, bg = map(_f32, (colors, opacities, map_opacities, background))
        xy, dp, cn = map(_f32, (xys, depths, conics))
        rd, cum = _i32(radii), _i32(cum_tiles_hit)
        Bt = max(B, 1)
        geom_rows = Bt * n
        if xy.numel() != 2 * geom_rows:
            raise ValueError(f"xys has {xy.numel() // 2} rows, expected {geom_rows}")
        final_Ts = torch.empty((Bt * img_h, img_w), device=dev, dtype=torch.float32)
        final_idx = torch.empty((Bt * img_h, img_w), device=dev, dtype=torch.int32)
        out_img = torch.empty((Bt * img_h, img_w, 3), device=dev, dtype=torch.float32)
        out_depth = (torch.empty((Bt * img_h, img_w), device=dev, dtype=torch.float32)
                     if with_depth else None)
        p = _lib.ptr
        args = [p(col), col.numel() // 3, p(op), op.numel(), p(mo), mo.numel(), p(bg),
                bg.numel() // 3, p(xy), p(dp), p(rd), p(cn), p(cum), geom_rows, n, img_h, img_w,
                Bt * img_h, key_bits, p(final_Ts), p(final_idx), p(out_img)]
        with torch.cuda.device(dev):
            if with_depth:
                rc = lib.splax_rasterize_depth(*args, p(out_depth), _lib.stream_of(col))
            else:
                rc = lib.splax_rasterize(*args, _lib.stream_of(col))
        _lib.check(rc)
        # the backward reuses this sort: autograd's version counters guarantee that the saved
        # inputs are unchanged when it runs
        ctx.sort_token = lib.splax_last_sort_token()
        ctx.save_for_backward(col, op, mo, bg, xy, dp, rd, cn, cum, final_Ts, final_idx)
        ctx.statics = (n, img_h, img_w, B, with_depth, key_bits)
        ctx.shapes = (colors.shape, opacities.shape, xys.shape, depths.shape, conics.shape)
        ctx.mark_non_differentiable(final_Ts, final_idx)
        # the residual outputs get no zero-filled cotangents in the backward
        ctx.set_materialize_grads(False)
        lead = (B, img_h, img_w) if B else (img_h, img_w)
        img = out_img.view(*lead, 3)
        if with_depth:
            return img, out_depth.view(*lead), final_Ts, final_idx
        return img, final_Ts, final_idx

    @staticmethod
    def backward(ctx, v_img, *rest):
        col, op, mo, bg, xy, dp, rd, cn, cum, final_Ts, final_idx = ctx.saved_tensors
        n, img_h, img_w, B, with_depth, key_bits = ctx.statics
        dev = col.device
        Bt = max(B, 1)
        rows = Bt * n
        lib = _lib.load()
        vo = (_f32(v_img) if v_img is not None
              else torch.zeros((Bt * img_h, img_w, 3), device=dev, dtype=torch.float32))
        # colours / opacities shared by the images get their gradient summed in-kernel
        fold_c = bool(B) and col.numel() // 3 == n
        fold_o = bool(B) and op.numel() == n
        v_colors = torch.empty((n if fold_c else rows, 3), device=dev, dtype=torch.float32)
        v_opac = torch.empty((n if fold_o else rows,), device=dev, dtype=torch.float32)
        v_xy = torch.empty((rows, 2), device=dev, dtype=torch.float32)
        v_conic = torch.empty((rows, 3), device=dev, dtype=torch.float32)
        vd, v_depths = None, None
        if with_depth:
            v_dimg = rest[0]
            vd = (_f32(v_dimg) if v_dimg is not None
                  else torch.zeros((Bt * img_h, img_w), device=dev, dtype=torch.float32))
            v_depths = torch.empty((rows,), device=dev, dtype=torch.float32)
        p = _lib.ptr
        with torch.cuda.device(dev):
            lib.splax_reuse_sort(ctx.sort_token)
            rc = lib.splax_rasterize_bwd_ex(
                p(col), col.numel() // 3, p(op), op.numel(), p(mo), mo.numel(), p(bg),
                bg.numel() // 3, p(xy), p(dp), p(rd), p(cn), p(cum), rows, p(final_Ts),
                p(final_idx), p(vo), vo.numel() // (3 * img_w), p(vd),
                0 if vd is None else vd.numel() // img_w, n, img_h, img_w, rows, key_bits,
                int(fold_c), int(fold_o), p(v_colors), p(v_opac), p(v_xy), p(v_conic),
                p(v_depths), _lib.stream_of(col))
        _lib.check(rc)
        cs, os_, xs, ds, ks = ctx.shapes

        def fold(g, shape, width):
            if B and g.numel() // width != torch.Size(shape).numel() // width:
                g = g.view(Bt, -1).sum(0)
            return g.reshape(shape)

        g_depths = v_depths.reshape(ds) if v_depths is not None else None
        return (fold(v_colors, cs, 3), fold(v_opac, os_, 1), None, None, v_xy.reshape(xs),
                g_depths, None, v_conic.reshape(ks), None, None, None, None, None, None, None)


def _geometry_batch(xys: torch.Tensor, n: int) -> int:
    rows = xys.numel() // 2
    if rows % n != 0:
        raise ValueError(f"xys has {rows} rows, not a multiple of n={n}")
    return 0 if xys.dim() <= 2 else rows // n


def _call(colors, opacities, background, xys, depths, radii, conics, cum_tiles_hit, img_shape,
          map_opacities, with_depth):
    n = colors.shape[-2]
    H, W = img_shape
    B = _geometry_batch(xys, n)
    if map_opacities is None:
        map_opacities = opacities
    key_bits = _sort.key_bits_for(max(B, 1), H, W)
    return _RasterizeFn.apply(colors, opacities.reshape(-1), map_opacities.reshape(-1),
                              background.reshape(-1, 3), xys, depths, radii, conics,
                              cum_tiles_hit, int(n), int(H), int(W), int(B), bool(with_depth),
                              int(key_bits))


def rasterize(colors, opacities, background, xys, depths, radii, conics, cum_tiles_hit, *,
              img_shape: tuple[int, int], map_opacities=None) -> torch.Tensor:
    """Blend projected gaussians into an (H, W, 3) image (a leading B for batched geometry).

    Differentiable with respect to colors, opacities, xys and conics (splax/_rasterize/
    _rasterize.py:24-60); background, depths, radii and cum_tiles_hit are not differentiated.
    ``map_opacities`` (default: ``opacities``) drives the tile walk, as in antialiased mode.
    """
    img, _, _ = _call(colors, opacities, background, xys, depths, radii, conics, cum_tiles_hit,
                      img_shape, map_opacities, False)
    return img


def rasterize_depth(colors, opacities, background, xys, depths, radii, conics, cum_tiles_hit, *,
                    img_shape: tuple[int, int], map_opacities=None):
    """Blend into an image and the alpha-blended expected depth map (splax/_rasterize/
    _rasterize.py:63-99); the depth map is (H, W) (a leading B for batched geometry) and its
    cotangent flows back to the depths."""
    img, depth, _, _ = _call(colors, opacities, background, xys, depths, radii, conics,
                             cum_tiles_hit, img_shape, map_opacities, True)
    return img, depth
