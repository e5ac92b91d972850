"""Differentiable projection stage (splax/_project/_project.py), backed by libsplax_b200.

``project`` keeps the reference's signature and returns the same six outputs. The custom vjp
of the reference becomes a ``torch.autograd.Function``: one backward kernel computes every
gradient (means, scales, quaternions, viewmat, transforms) in a single pass and autograd keeps
what it needs. Opacities drive the integer tile counts only and get no gradient here.

Batching follows the reference's ``vmap_method="expand_dims"`` contract: every operand is
either shared (no leading batch axis) or carries one leading batch axis of size B; viewmats
are (4,4) or (B,4,4). One launch covers the whole batch and ``cum_tiles_hit`` is the global
inclusive scan over all B*N pairs. Gradients of shared operands are summed over the batch.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from splax_b200 import _lib


def _rows_batch(x: torch.Tensor, n: int, width: int) -> int:
    """Leading batch of a per-gaussian operand: 0 when shared, else B."""
    total = x.numel() // width
    if total == n:
        return 0
    if total % n != 0:
        raise ValueError(f"operand with {x.numel()} elements does not hold n={n} rows of {width}")
    return total // n


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.detach().to(torch.float32).contiguous()


def batch_size(n: int, means3d, scales, quats, viewmat, opacities, transforms=None) -> int:
    """B of a projection call (0 when nothing is batched)."""
    bs = {_rows_batch(means3d, n, 3), _rows_batch(scales, n, 3), _rows_batch(quats, n, 4),
          _rows_batch(opacities, n, 1)}
    if viewmat.dim() == 3:
        bs.add(viewmat.shape[0])
    if transforms is not None and transforms.dim() == 4:
        bs.add(transforms.shape[0])
    bs.discard(0)
    if len(bs) > 1:
        raise ValueError(f"inconsistent batch sizes {sorted(bs)}")
    return bs.pop() if bs else 0


class _ProjectFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3d, scales, quats_wxyz, viewmat, opac, transforms, tf_ids, n, img_h,
                img_w, fx, fy, cx, cy, glob_scale, clip_thresh, has_transforms, B, aa_eps):
        dev = _lib.require_cuda(means3d, scales, quats_wxyz, viewmat, opac)
        lib = _lib.load()
        m, s, q, vm, o = map(_f32, (means3d, scales, quats_wxyz, viewmat, opac))
        tf = _f32(transforms)
        ids = tf_ids.detach().to(torch.int32).contiguous()
        K = transforms.shape[-3]
        Bt = max(B, 1)
        total = Bt * n
        xys = torch.empty((total, 2), device=dev, dtype=torch.float32)
        depths = torch.empty((total,), device=dev, dtype=torch.float32)
        radii = torch.empty((total,), device=dev, dtype=torch.int32)
        conics = torch.empty((total, 3), device=dev, dtype=torch.float32)
        nth = torch.empty((total,), device=dev, dtype=torch.int32)
        cum = torch.empty((total,), device=dev, dtype=torch.int32)
        aa = aa_eps is not None
        rho = torch.empty((total if aa else 0,), device=dev, dtype=torch.float32)
        p = _lib.ptr
        args = [p(m), m.numel() // 3, p(s), s.numel() // 3, p(q), q.numel() // 4, p(vm),
                vm.numel() // 4, p(o), o.numel(), p(tf), tf.numel() // 16, p(ids), n, K,
                int(has_transforms), img_h, img_w, fx, fy, cx, cy, glob_scale, clip_thresh,
                total, p(xys), p(depths), p(radii), p(conics), p(nth), p(cum)]
        eps, eps2 = _aa_consts(aa_eps) if aa else (0.0, 0.0)
        with torch.cuda.device(dev):
            # quaternions stay scalar-first: the kernel reads wxyz directly
            rc = lib.splax_project_ex(*args, 1, eps, eps2, p(rho) if aa else None,
                                      _lib.stream_of(m))
        _lib.check(rc)
        lead = (B, n) if B else (n,)
        outs = (xys.view(*lead, 2), depths.view(*lead, 1), radii.view(*lead, 1),
                conics.view(*lead, 3), nth.view(*lead, 1), cum.view(*lead, 1),
                rho.view(*lead) if aa else rho)
        ctx.save_for_backward(m, s, q, vm, tf, ids, radii, conics)
        ctx.statics = (n, fx, fy, glob_scale, has_transforms, B, K, aa_eps)
        ctx.shapes = (means3d.shape, scales.shape, quats_wxyz.shape, viewmat.shape,
                      transforms.shape)
        ctx.mark_non_differentiable(outs[2], outs[4], outs[5])
        if not aa:
            ctx.mark_non_differentiable(outs[6])
        # unused outputs get no zero-filled cotangents; the kernel treats NULL as zero
        ctx.set_materialize_grads(False)
        return outs

    @staticmethod
    def backward(ctx, v_xys, v_depths, _v_radii, v_conics, _v_nth, _v_cum, v_rho):
        m, s, q, vm, tf, ids, radii, conics = ctx.saved_tensors
        n, fx, fy, glob_scale, has_transforms, B, K, aa_eps = ctx.statics
        dev = m.device
        Bt = max(B, 1)
        total = Bt * n
        vxy = _f32(v_xys) if v_xys is not None else None
        vd = _f32(v_depths) if v_depths is not None else None
        vc = (_f32(v_conics) if v_conics is not None
              else torch.zeros((total, 3), device=dev, dtype=torch.float32))
        vr = _f32(v_rho) if (aa_eps is not None and v_rho is not None) else None
        # operands shared by the batch get their gradient summed over the images in-kernel
        fold = bool(B) and m.numel() // 3 == n and s.numel() // 3 == n and q.numel() // 4 == n
        grows = n if fold else total
        v_mean = torch.empty((grows, 3), device=dev, dtype=torch.float32)
        v_scale = torch.empty((grows, 3), device=dev, dtype=torch.float32)
        v_quat = torch.empty((grows, 4), device=dev, dtype=torch.float32)
        v_view = torch.empty((Bt, 4, 4), device=dev, dtype=torch.float32)
        v_tf = torch.empty((Bt, K, 4, 4), device=dev, dtype=torch.float32)
        p = _lib.ptr
        lib = _lib.load()
        eps, eps2 = _aa_consts(aa_eps) if vr is not None else (0.0, 0.0)
        with torch.cuda.device(dev):
            rc = lib.splax_project_bwd_ex(
                p(m), m.numel() // 3, p(s), s.numel() // 3, p(q), q.numel() // 4, p(vm),
                vm.numel() // 4, p(radii), radii.numel(), p(conics), conics.numel() // 3,
                p(vxy), total if vxy is None else vxy.numel() // 2,
                p(vd), total if vd is None else vd.numel(), p(vc), vc.numel() // 3,
                p(vr), total if vr is None else vr.numel(), eps, eps2, p(tf), tf.numel() // 16,
                p(ids), n, K, int(has_transforms), fx, fy, glob_scale, total, 1, int(fold),
                p(v_mean), p(v_scale), p(v_quat), p(v_view), p(v_tf), _lib.stream_of(m))
        _lib.check(rc)
        ms, ss, qs, vs, ts = ctx.shapes

        def fold_rows(g, shape, width):
            # shared operand not folded in-kernel: sum the per-image slots
            if B and g.numel() // width != (torch.Size(shape).numel() // width):
                g = g.view(Bt, -1).sum(0)
            return g.reshape(shape)

        g_tf = None
        if has_transforms and ctx.needs_input_grad[5]:
            g_tf = v_tf if len(ts) == 4 else v_tf.sum(0)
            g_tf = g_tf.reshape(ts)
        g_view = v_view if len(vs) == 3 else v_view.sum(0)
        return (fold_rows(v_mean, ms, 3), fold_rows(v_scale, ss, 3), fold_rows(v_quat, qs, 4),
                g_view.reshape(vs), None, g_tf, None, *([None] * 12))


# Read-only stand-ins for "no transforms" (a zero 4x4 matrix and a -1 id), made once per device:
# the kernels do not read them when has_transforms is 0, and making them on every call would put
# two fill kernels in front of each projection.
_NO_TRANSFORMS: dict = {}


def _no_transforms(dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    key = (dev.type, dev.index)
    got = _NO_TRANSFORMS.get(key)
    if got is None:
        got = (torch.zeros((1, 4, 4), device=dev, dtype=torch.float32),
               torch.full((1,), -1, device=dev, dtype=torch.int32))
        _NO_TRANSFORMS[key] = got
    return got


def _aa_consts(eps: float) -> tuple[float, float]:
    """eps and eps^2 as fp32 operands, rounded like the torch expression in
    ``opacity_compensation`` (a Python-float scalar times an fp32 tensor)."""
    e = float(torch.tensor(eps, dtype=torch.float32))
    e2 = float(torch.tensor(eps * eps, dtype=torch.float32))
    return e, e2


def project(
    mean3ds: torch.Tensor,
    scales: torch.Tensor,
    quats: torch.Tensor,
    viewmat: torch.Tensor,
    *,
    opacities: torch.Tensor,
    img_shape: tuple[int, int],
    f: tuple[float, float],
    c: tuple[float, float] | None = None,
    glob_scale: float = 1.0,
    clip_thresh: float = 0.01,
    gaussian_transforms: torch.Tensor | None = None,
    transform_ids: torch.Tensor | None = None,
    antialias_eps: float | None = None,
):
    """Project gaussians to screen space with the opacity-aware tile intersection.

    Mirrors ``splax.project`` (splax/_project/_project.py:25-92): quaternions are wxyz,
    ``c`` defaults to the image center, and the six outputs are the screen-space centers
    (N,2), depths (N,1), radii (N,1), conics (N,3), tile counts (N,1) and their global
    inclusive scan (N,1) -- each with a leading B when any operand is batched. The integer
    outputs are int32. With ``antialias_eps`` (not in the reference's signature; ``render``
    passes 0.3 when antialiased) the kernel also returns, as a seventh output, the per-pair
    compensation ``opacity_compensation(conics, radii, eps)`` computed in the same launch, and
    its gradient reaches the conics inside the backward kernel.
    """
    n = mean3ds.shape[-2]
    if c is None:
        c = (img_shape[1] / 2, img_shape[0] / 2)
    has_transforms = gaussian_transforms is not None
    dev = mean3ds.device
    if not has_transforms:
        gaussian_transforms, transform_ids = _no_transforms(dev)
    elif transform_ids is None:
        raise ValueError("gaussian_transforms needs transform_ids")
    B = batch_size(n, mean3ds, scales, quats, viewmat, opacities,
                   gaussian_transforms if has_transforms else None)
    H, W = img_shape
    outs = _ProjectFn.apply(
        mean3ds, scales, quats, viewmat, opacities.reshape(-1), gaussian_transforms,
        transform_ids, int(n), int(H), int(W), float(f[0]), float(f[1]), float(c[0]),
        float(c[1]), float(glob_scale), float(clip_thresh), bool(has_transforms), int(B),
        None if antialias_eps is None else float(antialias_eps))
    return outs if antialias_eps is not None else outs[:6]


def opacity_compensation(conics: torch.Tensor, radii: torch.Tensor, eps: float = 0.3) -> torch.Tensor:
    """Mip-Splatting anti-aliased opacity compensation (splax/_project/_project.py:95-117).

    rho = sqrt(clip(1 - eps (a + c) + eps^2 (a c - b^2), 0, 1)) from the dilated conic, 1 for
    culled gaussians. Plain torch ops, so its gradient reaches the conics through autograd.
    Returns one factor per gaussian (with the conics' leading batch).
    """
    a, b, cc = conics[..., 0], conics[..., 1], conics[..., 2]
    rho2 = 1.0 - eps * (a + cc) + (eps * eps) * (a * cc - b * b)
    rho = torch.sqrt(torch.clamp(rho2, 0.0, 1.0))
    return torch.where(radii.reshape(rho.shape) > 0, rho, torch.ones_like(rho))


def transform_ids(n: int, slices: Sequence[tuple[int, int]], device=None) -> torch.Tensor:
    """Per-gaussian transform index (splax/_project/_project.py:120-136); -1 for static ones.

    Slices must be static, non-overlapping and inside [0, n); violations raise ValueError.
    """
    for k, (start, stop) in enumerate(slices):
        if not (0 <= start < stop <= n):
            raise ValueError(f"gaussian slice {k} = [{start}, {stop}) outside [0, {n})")
    ordered = sorted(slices)
    for (_, prev_stop), (start, _) in zip(ordered, ordered[1:]):
        if start < prev_stop:
            raise ValueError(f"gaussian slices overlap: {list(slices)}")
    ids = torch.full((n,), -1, dtype=torch.int32, device=device)
    for k, (start, stop) in enumerate(slices):
        ids[start:stop] = k
    return ids
