/*
 * CPU restatement of the splax splatting hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This library is the parity checker for the CUDA path in splax_b200/csrc. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load it. The product
 * path never calls it and has no CPU fallback.
 *
 * It restates, in plain C11 fp32 (no fast-math, no FMA contraction), the Warp kernels of
 * amacati/splax:
 *   projection           splax/_project/_kernels.py:122-248 (+ helpers :609-664)
 *   ellipse tile walk    splax/_intersect.py:47-183
 *   global scan          splax/_project/_kernels.py:104-107 (inclusive int32 scan)
 *   depth min/max        splax/_rasterize/_sort/_kernels.py:31-73
 *   key width choice     splax/_rasterize/_sort/_sort.py:23-66
 *   key emission         splax/_rasterize/_sort/_kernels.py:76-211
 *   radix sort           warp.utils.radix_sort_pairs, a stable ascending (signed) pair sort
 *   bin edges            splax/_rasterize/_sort/_kernels.py:214-269
 *   forward blend        splax/_rasterize/_kernels.py:102-205 and the depth twin :277-380
 *   backward blend       splax/_rasterize/_kernels.py:530-665, :935-1076, vjps :1212-1302
 *   projection backward  splax/_project/_kernels.py:356-606
 *
 * Parity pin: warp-lang 1.15.0 and jax 0.11.0 (the reference's pinned runtime) are not
 * installable here. The reference's kernels are Warp-DSL Python, though, and
 * tests/golden/make_reference_fixtures.py executes them unmodified under a CPU stand-in for
 * warp's API (tests/golden/warp_standin.py): _project_warp with _project_kernel and the
 * ellipse walk, sort_and_bin with its key, sort and bin kernels, and _project_bwd_warp. On
 * those fixtures this restatement reproduces projection, keys, sorted ids and bins bit for bit
 * and the per-pair projection gradients bit for bit (tests/test_reference_fixtures.py). The
 * pin holds under the stand-in's builtin semantics (IEEE fp32 without contraction, this
 * file's logarithm, the standard quaternion matrix), which Warp's own fast-math native code
 * may differ from by an ulp. The blend kernels use Warp tile primitives that the stand-in does
 * not run; they are pinned to the reference's known-answer tests (tests/test_depth_reg.py:
 * 75-107, tests/test_antialiased.py:71-97), invariants (tests/test_warp_rasterize.py:433-487,
 * tests/test_warp_batch.py:102-126) and an independent float64 numpy restatement
 * (tests/golden/make_golden.py).
 *
 * Determinism contract shared with the CUDA path: every float operation that feeds an
 * integer output (tile counts, radii, keys, bins) uses IEEE-754 single precision +,-,*,/,sqrt
 * in the order written here, with no fused multiply-add, and the logarithm is splat_logf
 * below (an atanh series, not the platform libm), so the CUDA projection and emission
 * kernels reproduce these integers bit for bit.
 */
#ifndef SPLAT_ORACLE_H
#define SPLAT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* constants of splax/_intersect.py:17-20 and splax/_rasterize/_kernels.py:188-192 */
#define ORC_BLOCK_WIDTH 16

/* Deterministic natural logarithm shared (as a restatement) with the CUDA kernels. */
float orc_logf(float x);

/* Projection forward: K1 + K2 (splax/_project/_kernels.py:31-107, 122-248).
 * *_rows is each input's leading length (n for a shared input, B*n for a batched one);
 * viewmat_rows is 4 or 4*B; transforms_rows is K or B*K. total = B*n output rows. */
void orc_project(const float *means3d, int64_t means_rows, const float *scales,
                 int64_t scales_rows, const float *quats_xyzw, int64_t quats_rows,
                 const float *viewmat, int64_t viewmat_rows, const float *opacities,
                 int64_t opac_rows, const float *transforms, int64_t transforms_rows,
                 const int32_t *transform_ids, int32_t n, int32_t num_transforms,
                 int32_t has_transforms, int32_t img_h, int32_t img_w, float fx, float fy,
                 float cx, float cy, float glob_scale, float clip_thresh, int64_t total,
                 float *xys, float *depths, int32_t *radii, float *conics,
                 int32_t *num_tiles_hit, int32_t *cum_tiles_hit, int nthreads);

/* Key width decision of splax/_rasterize/_sort/_sort.py:51-66.
 * key_bits_request: 0 = the reference's default rule (depth_bits >= 16), 32 or 64 = forced.
 * Returns 32 or 64, or -1 on key overflow (upper bits > 32 on the 64-bit path). */
int orc_key_bits(int32_t B, int32_t img_h, int32_t img_w, int key_bits_request,
                 int32_t *tile_n_bits, int32_t *depth_bits);

/* sort_and_bin (splax/_rasterize/_sort/_sort.py:29-171) over the flat B*n projection.
 * gaussian_ids and keys (optional, may be NULL) need num_intersects entries, where
 * num_intersects = cum_tiles_hit[B*n-1]; tile_bins needs 2*B*T int32.
 * Returns 0, or -1 on key overflow, or -2 if the emitted count disagrees with cum. */
int orc_sort_and_bin(const float *xys, const float *depths, const int32_t *radii,
                     const float *conics, const float *map_opacities, int64_t map_opac_rows,
                     const int32_t *cum_tiles_hit, int32_t n, int32_t B, int32_t img_h,
                     int32_t img_w, int key_bits_request, int32_t *gaussian_ids,
                     int64_t *keys, int32_t *tile_bins, int32_t *used_key_bits,
                     int nthreads);

/* Emission only (K5), unsorted, at the cum offsets; for the emit == count invariant. */
int orc_map_intersects(const float *xys, const float *depths, const int32_t *radii,
                       const float *conics, const float *map_opacities, int64_t map_opac_rows,
                       const int32_t *cum_tiles_hit, int32_t n, int32_t B, int32_t img_h,
                       int32_t img_w, int key_bits, int64_t *keys, int32_t *gaussian_ids);

/* Forward blend (K8, or K9 when out_depth != NULL) after sort_and_bin.
 * B = number of output images. flags (optional) receives, per pixel, 1 when one of the
 * pixel's threshold decisions (alpha vs 1/255, transmittance vs 1e-4, sign of sigma) lies
 * within rounding distance of its boundary, so that a different but correct fp32 evaluation
 * order may decide it the other way. */
int orc_rasterize(const float *colors, int64_t color_rows, const float *opacities,
                  int64_t opac_rows, const float *map_opacities, int64_t map_opac_rows,
                  const float *background, int64_t bg_rows, const float *xys,
                  const float *depths, const int32_t *radii, const float *conics,
                  const int32_t *cum_tiles_hit, int32_t n, int32_t B, int32_t img_h,
                  int32_t img_w, int key_bits_request, float *final_Ts, int32_t *final_idx,
                  float *out_img, float *out_depth, uint8_t *flags, int nthreads);

/* Backward blend (K10/K11, or K12/K13 when v_out_depth != NULL).
 * B_out = images the cotangent covers, B_geom = renders the geometry covers (1 or B_out).
 * vout_rows / vdepth_rows are the cotangents' row counts (H or B_out*H).
 * Outputs have B_out*n rows and are overwritten (accumulated in double, then rounded). */
int orc_rasterize_bwd(const float *colors, int64_t color_rows, const float *opacities,
                      int64_t opac_rows, const float *map_opacities, int64_t map_opac_rows,
                      const float *background, int64_t bg_rows, const float *xys,
                      const float *depths, const int32_t *radii, const float *conics,
                      const int32_t *cum_tiles_hit, const float *final_Ts,
                      const int32_t *final_idx, const float *v_out_img, int64_t vout_rows,
                      const float *v_out_depth, int64_t vdepth_rows, int32_t n, int32_t B_out,
                      int32_t B_geom, int32_t img_h, int32_t img_w, int key_bits_request,
                      float *v_colors, float *v_opacity, float *v_xy, float *v_conic,
                      float *v_depths, int nthreads);

/* Projection backward (K14, splax/_project/_kernels.py:257-606). B = v_mean rows / n. */
void orc_project_bwd(const float *means3d, int64_t means_rows, const float *scales,
                     int64_t scales_rows, const float *quats_xyzw, int64_t quats_rows,
                     const float *viewmat, int64_t viewmat_rows, const int32_t *radii,
                     int64_t radii_rows, const float *conics, int64_t conics_rows,
                     const float *v_xy, int64_t vxy_rows, const float *v_depth,
                     int64_t vdepth_rows, const float *v_conic, int64_t vconic_rows,
                     const float *transforms, int64_t transforms_rows,
                     const int32_t *transform_ids, int32_t n, int32_t num_transforms,
                     int32_t has_transforms, float fx, float fy, float glob_scale, int32_t B,
                     float *v_mean3d, float *v_scale, float *v_quat, float *v_viewmat,
                     float *v_transforms, int nthreads);

/* Ellipse-walk tile count per gaussian for given screen-space geometry (test helper). */
void orc_tile_counts(const float *xys, const int32_t *radii, const float *conics,
                     const float *map_opacities, int64_t opac_rows, int64_t total,
                     int32_t img_h, int32_t img_w, int32_t *counts);

/* Work counters of the last orc_rasterize / orc_rasterize_bwd call (roofline units):
 * [0] intersections I, [1] forward evaluations E_f, [2] forward contributions,
 * [3] backward evaluations E_b, [4] backward contributions C_b. */
void orc_counters(int64_t out[5]);

#ifdef __cplusplus
}
#endif
#endif
