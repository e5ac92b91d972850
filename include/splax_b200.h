/*
 * splax_b200 C ABI: the splatting hot path of amacati/splax as plain C entry points.
 *
 * Each entry point replaces one of the XLA FFI targets the reference builds with
 * warp.jax_callable and wraps in nested_vmap (splax/_batching.py:32-115). Arguments follow
 * the Warp wrappers' order and meaning; every array is a device pointer plus its leading
 * length ("rows") as the reference's FFI bridge sees it after collapsing vmap batches
 * (vmap_method="expand_dims"): a per-gaussian input has n rows when shared across the batch
 * and B*n rows when batched, a viewmat 4 or 4*B rows, a transform stack K or B*K matrices,
 * an image B*H rows. Inner widths are fixed: xys 2, conics 3, colors 3, quats 4 (xyzw),
 * matrices 4x4 row-major, images W*3 (colour) or W (scalars). All floats are fp32.
 *
 * Streams: all work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream)
 * of the current CUDA device. Rasterize entry points block the calling thread once, on the
 * intersection-count readback, exactly like the reference (splax/_cache.py:130-155), so they
 * cannot be captured into a CUDA graph.
 *
 * Scratch: the sort keys and values (2 x 1.25 x intersections), tile bins, per-image depth
 * ranges and packed blend records are owned by the library per device, grow-only, and
 * dropped when the (B, n, tiles) signature changes or on splax_clear_cache()
 * (splax/_cache.py:52-90, 158-164). Calls that overlap on the GPU on one device (two
 * streams at once) share that scratch and must be serialised by the caller.
 *
 * Errors: a nonzero return is an SPLAX_ERR_* code; splax_last_error() gives the message of
 * the calling thread's last failure. Device-side checks (bounded spin-waits, emitted count vs
 * cum_tiles_hit, negative 64-bit depth keys, int32 count overflow) raise a device error word
 * that the next count readback (or splax_check_device_errors) reports.
 */
#ifndef SPLAX_B200_H
#define SPLAX_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPLAX_OK 0
#define SPLAX_ERR_INVALID_ARGUMENT 1 /* ValueError in the reference */
#define SPLAX_ERR_KEY_OVERFLOW 2     /* splax/_rasterize/_sort/_sort.py:61-66 (ValueError) */
#define SPLAX_ERR_OUT_OF_MEMORY 3
#define SPLAX_ERR_CUDA 4
#define SPLAX_ERR_DEVICE 5         /* device-side check failed, see splax_last_error() */
#define SPLAX_ERR_COUNT_OVERFLOW 6 /* intersections exceed the int32 range of the ABI */

/* Message of the calling thread's last failed call ("" if none). */
const char *splax_last_error(void);

/* Library version string. */
const char *splax_version(void);

/* FFI target "project": _project_warp, splax/_project/_kernels.py:31-107 (:110-119).
 * Writes xys (total,2), depths, radii, conics (total,3), num_tiles_hit and the global
 * inclusive scan cum_tiles_hit for total = B*n (camera, gaussian) pairs. */
int splax_project(const float *means3d, int64_t means3d_rows, const float *scales,
                  int64_t scales_rows, const float *quats_xyzw, int64_t quats_rows,
                  const float *viewmat, int64_t viewmat_rows, const float *opacities,
                  int64_t opacities_rows, const float *gaussian_transforms,
                  int64_t transforms_rows, const int32_t *transform_ids, int32_t num_gaussians,
                  int32_t num_transforms, int32_t has_transforms, int32_t img_h, int32_t img_w,
                  float fx, float fy, float cx, float cy, float glob_scale, float clip_thresh,
                  int64_t total, float *xys, float *depths, int32_t *radii, float *conics,
                  int32_t *num_tiles_hit, int32_t *cum_tiles_hit, void *stream);

/* Projection forward that allocates nothing. No counterpart in the reference: same arguments
 * and outputs as splax_project, for callers that cannot let a library call cudaMalloc (an XLA
 * custom call in a JAX process whose allocator has reserved most of the GPU up front, or an
 * embedder with a fixed device-memory budget). Its scan scratch is a file-scope __device__
 * array of 128 KiB + 16 bytes, held by every GPU that loads the library until the process
 * exits, so total = B*n is limited to 16,777,216 pairs (larger calls fail with
 * SPLAX_ERR_INVALID_ARGUMENT). The first call on a device resolves the array's address; make
 * it before any stream capture. Calls share the array: calls overlapping on the GPU race.
 * Device-side errors (an intersection count past the int32 range, a scan wait that gave up)
 * land in the array's own error word, which is read back only when SPLAX_SYNC_CHECK=1 (the call
 * then synchronises the stream); otherwise they go unreported on this path. */
int splax_project_noalloc(const float *means3d, int64_t means3d_rows, const float *scales,
                          int64_t scales_rows, const float *quats_xyzw, int64_t quats_rows,
                          const float *viewmat, int64_t viewmat_rows, const float *opacities,
                          int64_t opacities_rows, const float *gaussian_transforms,
                          int64_t transforms_rows, const int32_t *transform_ids,
                          int32_t num_gaussians, int32_t num_transforms, int32_t has_transforms,
                          int32_t img_h, int32_t img_w, float fx, float fy, float cx, float cy,
                          float glob_scale, float clip_thresh, int64_t total, float *xys,
                          float *depths, int32_t *radii, float *conics, int32_t *num_tiles_hit,
                          int32_t *cum_tiles_hit, void *stream);

/* FFI target "project_bwd": _project_bwd_warp, splax/_project/_kernels.py:257-341 (:344-353).
 * B = out_rows / num_gaussians images; outputs v_mean3d (B*n,3), v_scale (B*n,3),
 * v_quat (B*n,4) xyzw, v_viewmat (4B,4), v_transforms (B*K,4,4), all overwritten. */
int splax_project_bwd(const float *means3d, int64_t means3d_rows, const float *scales,
                      int64_t scales_rows, const float *quats_xyzw, int64_t quats_rows,
                      const float *viewmat, int64_t viewmat_rows, const int32_t *radii,
                      int64_t radii_rows, const float *conics, int64_t conics_rows,
                      const float *v_xy, int64_t v_xy_rows, const float *v_depth,
                      int64_t v_depth_rows, const float *v_conic, int64_t v_conic_rows,
                      const float *gaussian_transforms, int64_t transforms_rows,
                      const int32_t *transform_ids, int32_t num_gaussians, int32_t num_transforms,
                      int32_t has_transforms, float fx, float fy, float glob_scale,
                      int64_t out_rows, float *v_mean3d, float *v_scale, float *v_quat,
                      float *v_viewmat, float *v_transforms, void *stream);

/* Projection with options (no FFI counterpart in the reference, whose JAX side rolls the
 * quaternions to xyzw and computes opacity_compensation, splax/_project/_project.py:95-117,
 * from the projection's outputs): splax_project's arguments, then quats_wxyz (1: quaternions
 * stored scalar-first, read without a reorder pass), and the antialiasing compensation folded
 * into the same launch -- with rho non-NULL, rho (total,) receives
 * sqrt(clip(1 - eps (a + c) + eps2 (a c - b^2), 0, 1)) of each pair's conic, 1 when culled;
 * eps is the 0.3 px^2 dilation and eps2 = eps*eps as the caller rounds it to fp32. */
int splax_project_ex(const float *means3d, int64_t means3d_rows, const float *scales,
                     int64_t scales_rows, const float *quats, int64_t quats_rows,
                     const float *viewmat, int64_t viewmat_rows, const float *opacities,
                     int64_t opacities_rows, const float *gaussian_transforms,
                     int64_t transforms_rows, const int32_t *transform_ids,
                     int32_t num_gaussians, int32_t num_transforms, int32_t has_transforms,
                     int32_t img_h, int32_t img_w, float fx, float fy, float cx, float cy,
                     float glob_scale, float clip_thresh, int64_t total, float *xys,
                     float *depths, int32_t *radii, float *conics, int32_t *num_tiles_hit,
                     int32_t *cum_tiles_hit, int32_t quats_wxyz, float aa_eps, float aa_eps2,
                     float *rho, void *stream);

/* Backward of splax_project_ex: splax_project_bwd's arguments, with
 * - v_xy / v_depth may be NULL (zero cotangents; their rows are ignored);
 * - v_rho (n or B*n rows, or NULL): the cotangent of rho, chained through d rho / d conic into
 *   the conic cotangent (zero where the clip is active or the pair is culled), with the same
 *   eps and eps2;
 * - quats_wxyz: quats and v_quat stored scalar-first;
 * - fold_batch (1): v_mean3d, v_scale and v_quat get n rows, each the sum over the B images
 *   (what a caller sums for operands shared by the batch); needs n-row means, scales, quats. */
int splax_project_bwd_ex(const float *means3d, int64_t means3d_rows, const float *scales,
                         int64_t scales_rows, const float *quats, int64_t quats_rows,
                         const float *viewmat, int64_t viewmat_rows, const int32_t *radii,
                         int64_t radii_rows, const float *conics, int64_t conics_rows,
                         const float *v_xy, int64_t v_xy_rows, const float *v_depth,
                         int64_t v_depth_rows, const float *v_conic, int64_t v_conic_rows,
                         const float *v_rho, int64_t v_rho_rows, float aa_eps, float aa_eps2,
                         const float *gaussian_transforms, int64_t transforms_rows,
                         const int32_t *transform_ids, int32_t num_gaussians,
                         int32_t num_transforms, int32_t has_transforms, float fx, float fy,
                         float glob_scale, int64_t out_rows, int32_t quats_wxyz,
                         int32_t fold_batch, float *v_mean3d, float *v_scale, float *v_quat,
                         float *v_viewmat, float *v_transforms, void *stream);

/* FFI target "rasterize": _rasterize_warp, splax/_rasterize/_kernels.py:37-87 (:90-99).
 * geom_rows = rows of xys / depths / radii / conics / cum_tiles_hit (= B*n); out_rows = B*H.
 * key_bits: 0 = the reference's automatic width (splax/_rasterize/_sort/_sort.py:23-26),
 * 32 or 64 to force one, the role of the reference's monkeypatchable _use_32bit_keys hook.
 * Writes final_Ts (B*H,W), final_idx (B*H,W) and out_img (B*H,W,3). */
int splax_rasterize(const float *colors, int64_t colors_rows, const float *opacities,
                    int64_t opacities_rows, const float *map_opacities, int64_t map_opacities_rows,
                    const float *background, int64_t background_rows, const float *xys,
                    const float *depths, const int32_t *radii, const float *conics,
                    const int32_t *cum_tiles_hit, int64_t geom_rows, int32_t num_gaussians,
                    int32_t img_h, int32_t img_w, int64_t out_rows, int32_t key_bits,
                    float *final_Ts, int32_t *final_idx, float *out_img, void *stream);

/* FFI target "rasterize_depth": _rasterize_depth_warp, splax/_rasterize/_kernels.py:208-262
 * (:265-274). As splax_rasterize plus out_depth (B*H,W), the alpha-blended expected depth. */
int splax_rasterize_depth(const float *colors, int64_t colors_rows, const float *opacities,
                          int64_t opacities_rows, const float *map_opacities,
                          int64_t map_opacities_rows, const float *background,
                          int64_t background_rows, const float *xys, const float *depths,
                          const int32_t *radii, const float *conics, const int32_t *cum_tiles_hit,
                          int64_t geom_rows, int32_t num_gaussians, int32_t img_h, int32_t img_w,
                          int64_t out_rows, int32_t key_bits, float *final_Ts, int32_t *final_idx,
                          float *out_img, float *out_depth, void *stream);

/* FFI target "rasterize_bwd": _rasterize_bwd_warp, splax/_rasterize/_kernels.py:386-500
 * (:503-512). B_geom = geom_rows / n renders were sorted; B_out = grad_rows / n images
 * receive cotangents (B_out may exceed B_geom = 1: a shared render against B targets).
 * v_out_img has v_out_rows = H (broadcast) or B_out*H rows. Outputs (grad_rows rows):
 * v_colors (,3), v_opacity, v_xy (,2), v_conic (,3), overwritten. */
int splax_rasterize_bwd(const float *colors, int64_t colors_rows, const float *opacities,
                        int64_t opacities_rows, const float *map_opacities,
                        int64_t map_opacities_rows, const float *background,
                        int64_t background_rows, const float *xys, const float *depths,
                        const int32_t *radii, const float *conics, const int32_t *cum_tiles_hit,
                        int64_t geom_rows, const float *final_Ts, const int32_t *final_idx,
                        const float *v_out_img, int64_t v_out_rows, int32_t num_gaussians,
                        int32_t img_h, int32_t img_w, int64_t grad_rows, int32_t key_bits,
                        float *v_colors, float *v_opacity, float *v_xy, float *v_conic,
                        void *stream);

/* FFI target "rasterize_bwd_depth": _rasterize_bwd_depth_warp,
 * splax/_rasterize/_kernels.py:797-914 (:917-926). As splax_rasterize_bwd plus the depth
 * cotangent v_out_depth (v_out_depth_rows = H or B_out*H) and the output v_depths. */
int splax_rasterize_bwd_depth(const float *colors, int64_t colors_rows, const float *opacities,
                              int64_t opacities_rows, const float *map_opacities,
                              int64_t map_opacities_rows, const float *background,
                              int64_t background_rows, const float *xys, const float *depths,
                              const int32_t *radii, const float *conics,
                              const int32_t *cum_tiles_hit, int64_t geom_rows,
                              const float *final_Ts, const int32_t *final_idx,
                              const float *v_out_img, int64_t v_out_rows,
                              const float *v_out_depth, int64_t v_out_depth_rows,
                              int32_t num_gaussians, int32_t img_h, int32_t img_w,
                              int64_t grad_rows, int32_t key_bits, float *v_colors,
                              float *v_opacity, float *v_xy, float *v_conic, float *v_depths,
                              void *stream);

/* Rasterize backward with options (no FFI counterpart: the reference's JAX side sums the
 * per-image gradients of operands shared by the batch): the plain or depth variant (depth when
 * v_out_depth and v_depths are both non-NULL), and fold_colors / fold_opacity (1: v_colors /
 * v_opacity get n rows, each the sum over the images; needs n-row colors / opacities). */
int splax_rasterize_bwd_ex(const float *colors, int64_t colors_rows, const float *opacities,
                           int64_t opacities_rows, const float *map_opacities,
                           int64_t map_opacities_rows, const float *background,
                           int64_t background_rows, const float *xys, const float *depths,
                           const int32_t *radii, const float *conics,
                           const int32_t *cum_tiles_hit, int64_t geom_rows,
                           const float *final_Ts, const int32_t *final_idx,
                           const float *v_out_img, int64_t v_out_rows, const float *v_out_depth,
                           int64_t v_out_depth_rows, int32_t num_gaussians, int32_t img_h,
                           int32_t img_w, int64_t grad_rows, int32_t key_bits,
                           int32_t fold_colors, int32_t fold_opacity, float *v_colors,
                           float *v_opacity, float *v_xy, float *v_conic, float *v_depths,
                           void *stream);

/* Reuse of the forward's sort by its backward (the reference re-sorts in every backward,
 * splax/_rasterize/_kernels.py:422-424; the sort is deterministic, so reusing it gives identical
 * results). splax_last_sort_token() returns the token of the sort done by the calling thread's
 * last splax_rasterize / splax_rasterize_depth call (-1 if none). splax_reuse_sort(token) arms
 * it for the calling thread's next backward call, which then skips its sort_and_bin when the
 * token is still the device's most recent sort and every geometry / opacity / colour pointer,
 * length and static is identical; otherwise it sorts as usual. Arm it only when the forward's
 * input buffers are unchanged since the forward. */
int64_t splax_last_sort_token(void);
void splax_reuse_sort(int64_t token);

/* sort_and_bin, splax/_rasterize/_sort/_sort.py:29-171, exposed for parity tests: copies
 * the sorted flat gaussian ids (capacity gaussian_ids_cap) and the (B*T) int2 tile bins into
 * caller buffers, and optionally the sorted keys (as int64, NULL to skip). Writes the
 * intersection count and the key width used. */
int splax_sort_and_bin(const float *xys, const float *depths, const int32_t *radii,
                       const float *conics, const float *map_opacities,
                       int64_t map_opacities_rows, const int32_t *cum_tiles_hit,
                       int32_t num_gaussians, int32_t num_images, int32_t img_h, int32_t img_w,
                       int32_t key_bits, int32_t *gaussian_ids, int64_t gaussian_ids_cap,
                       int64_t *sorted_keys, int32_t *tile_bins, int64_t *num_intersects,
                       int32_t *used_key_bits, void *stream);

/* Fused mean-squared-error loss of a rendered image stack. No counterpart in the reference,
 * whose callers take the loss in JAX (the MSE objective of the benchmark configurations; the
 * training step of scripts/train_colmap.py:118-295): loss[0] = sum((img - target)^2) / denom
 * over `count` floats, one pass over both arrays. img, target and loss are device pointers.
 * Deterministic (fixed grid, fixed-order final sum in fp64). */
int splax_mse_loss(const float *img, const float *target, int64_t count, float denom,
                   float *loss, void *stream);

/* Gradient of splax_mse_loss: grad = v_loss[0] * 2 (img - target) / denom, where v_loss is the
 * incoming cotangent as a device float (no host synchronisation). grad may alias neither
 * input. */
int splax_mse_loss_bwd(const float *img, const float *target, int64_t count, float denom,
                       const float *v_loss, float *grad, void *stream);

/* Fused photometric loss of the batched training step, (1 - lambda) L1 + lambda D-SSIM, for
 * B RGB images (B, H, W, 3) against targets of the same shape (device pointers). No
 * counterpart in the reference, whose training step takes it in JAX with dm_pix.ssim
 * (scripts/train_colmap.py:202-221): per view mean |img - gt| and 1 - ssim(img, gt), averaged
 * over views; SSIM with an 11-tap Gaussian window (sigma 1.5, VALID), k1 0.01, k2 0.03,
 * max_val 1, variances floored at eps_f32^2 and the covariance clamped to sqrt(var var).
 * views_total is the number of views over all ranks (B on one GPU): the loss written is this
 * rank's share, so the shares of all ranks add up to the loss. Needs H, W >= 11.
 * Deterministic (fixed-order fp64 partial sums). */
int splax_l1_dssim_loss(const float *img, const float *target, int32_t B, int32_t H, int32_t W,
                        int32_t views_total, float ssim_lambda, float *loss, void *stream);

/* Gradient of splax_l1_dssim_loss with respect to img, scaled by the cotangent v_loss[0] (a
 * device float, no host synchronisation); grad has img's shape and may alias neither input. */
int splax_l1_dssim_loss_bwd(const float *img, const float *target, int32_t B, int32_t H,
                            int32_t W, int32_t views_total, float ssim_lambda,
                            const float *v_loss, float *grad, void *stream);

/* splax_l1_dssim_loss and its gradient for a unit cotangent (v_loss = 1) in one pass: the
 * training step's loss and gradient together, at about the cost of the gradient alone. loss:
 * one device float; grad: img's shape, aliasing neither input. Scale grad by the cotangent when
 * it is not 1. */
int splax_l1_dssim_loss_and_grad(const float *img, const float *target, int32_t B, int32_t H,
                                 int32_t W, int32_t views_total, float ssim_lambda, float *loss,
                                 float *grad, void *stream);

/* Fused per-parameter Adam update, in place, of num_arrays fp32 parameter arrays (device
 * pointers in host arrays: params, grads, first / second moments, element counts, learning
 * rates). No counterpart in the reference, whose training step uses optax.adam per group
 * (scripts/train_colmap.py:639-645); the update is optax's scale_by_adam then -lr:
 * m = (1 - b1) g + b1 m, v = (1 - b2) g^2 + b2 v, p -= lr (m / (1 - b1^step)) /
 * (sqrt(v / (1 - b2^step)) + eps), with step >= 1 the update count after this step. */
int splax_adam_step(int32_t num_arrays, float *const *params, const float *const *grads,
                    float *const *exp_avg, float *const *exp_avg_sq, const int64_t *sizes,
                    const float *lrs, int32_t step, float b1, float b2, float eps, void *stream);

/* Sum all-reduce, in place, of n fp32 values held in a symmetric buffer by each of `world`
 * ranks (one process per GPU, all on one NVSwitch fabric), through NVLink SHARP: multicast is
 * the buffer's multicast address (16-byte aligned); flag_ptrs is a host array of `world`
 * device pointers, rank q's uint64[world] barrier flags inside its copy of the buffer (zero
 * before the first call). One call runs an entry barrier with `epoch`, the reduction of this
 * rank's shard (multimem.ld_reduce + multimem.st) and an exit barrier with epoch + 1, so epochs
 * advance by 2 per call, identically on every rank. A barrier that waits past its bound sets
 * bit 5 in *err (device word) and returns; from then on, while *err is nonzero, every launch of
 * this call and of later calls returns without touching peer or multicast memory, so the
 * caller must read *err and stop the run (the exchange is not restartable in place). No
 * counterpart in the reference, which has no
 * multi-device path: it replaces the psum of the gaussian gradients over a camera mesh that
 * a shard_map data-parallel training step would issue. */
int splax_nvls_allreduce_f32(float *multicast, void *const *flag_ptrs, int32_t rank,
                             int32_t world, int64_t n, uint64_t epoch, uint32_t *err,
                             void *stream);

/* The training step's gradient exchange fused with its Adam update, for the same symmetric
 * setup as splax_nvls_allreduce_f32: grad_mc and param_mc are the multicast addresses of two
 * symmetric buffers of n floats (the gradients, and the parameters whose local copy is
 * param_local), split into num_groups (1..8) consecutive parameter groups of group_sizes[k]
 * elements and learning rate lrs[k] (host arrays). Each rank sums its shard of the gradients
 * through the switch, applies Adam (splax_adam_step's update, step >= 1 after this update) with
 * its shard of the moments, exp_avg / exp_avg_sq of splax_nvls_adam_shard_len floats (zero
 * before the first step), and writes the updated parameters into every rank's copy; entry and
 * exit barriers use epoch and epoch + 1 on flag_ptrs (one flag array, as above). No counterpart
 * in the reference: it replaces the psum followed by optax.adam of a sharded training step. */
int splax_nvls_adam_step(const float *grad_mc, float *param_mc, const float *param_local,
                         float *exp_avg, float *exp_avg_sq, int64_t n, int32_t num_groups,
                         const int64_t *group_sizes, const float *lrs, int32_t step, float b1,
                         float b2, float eps, void *const *flag_ptrs, int32_t rank,
                         int32_t world, uint64_t epoch, uint32_t *err, void *stream);

/* Length (floats) of this rank's shard of the moments for splax_nvls_adam_step. */
int splax_nvls_adam_shard_len(int64_t n, int32_t rank, int32_t world, int64_t *len);

/* load_ply, splax/io.py:78-98, first half: parse a 3DGS .ply header and report its vertex
 * count (host only, no GPU work). Binary little-endian files whose first element is `vertex`
 * with scalar properties, the fields x y z scale_0..2 rot_0..3 f_dc_0..2 opacity in float32. */
int splax_ply_info(const char *path, int64_t *num_vertices);

/* load_ply, second half: stream the vertex records to the GPU and decode them into the five
 * render-space arrays (device pointers): means (n,3), scales = exp(scale) (n,3), quats =
 * rot / |rot| wxyz (n,4), colors = clip(f_dc * C0 + 0.5, 0, 1) (n,3), opacities =
 * sigmoid(opacity) (n,). num_vertices must be splax_ply_info's count. */
int splax_ply_load(const char *path, int64_t num_vertices, float *means, float *scales,
                   float *quats, float *colors, float *opacities, void *stream);

/* clear_cache, splax/_cache.py:158-164: release the scratch of every device. */
void splax_clear_cache(void);

/* Inspection of the current device's scratch entry (the reference's _scratch_cache, read by
 * tests/test_warp_rasterize.py:350,358): out[0] sort capacity, [1] key width (32/64, 0 when
 * empty), [2] bytes held, [3..5] signature (B, n, tiles). Returns the entries written. */
int splax_scratch_info(int64_t *out, int32_t out_len);

/* Synchronise `stream` and report any pending device-side error word. */
int splax_check_device_errors(void *stream);

/* Test hook for failure paths: after `successes` more device allocations, the next one fails
 * as out-of-memory (negative disables). Host-side only; no GPU fault is involved. */
void splax_debug_fail_alloc_after(int64_t successes);

/* Opt-in profiling (no counterpart in the reference, which has no built-in profiling):
 * `timing` records CUDA events around every launch sequence on its stream; `count_work`
 * switches the blend kernels to instrumented builds that count per-pixel evaluations and
 * contributions (the roofline's work units). Both default off. */
void splax_profile_enable(int32_t timing, int32_t count_work);

/* Restrict the timing of splax_profile_enable to some stages (no counterpart in the
 * reference): bit k set times stage k, in the order project_fwd, project_bwd, depth_minmax,
 * pair_keys, pair_sort, pair_scan, emit_keys, radix_sort, tile_bins, raster_fwd, raster_bwd,
 * loss, optim, allreduce (the names of splax_profile_report). Each timed stage adds two event
 * records to its stream; timing one stage keeps that cost out of the others. Default: all. */
void splax_profile_stages(uint32_t mask);

/* Zero the current device's timers and work counters. */
int splax_profile_reset(void);

/* JSON of the current device's per-kernel launches / kernels / milliseconds and work units
 * since the last reset; synchronises on pending timing events. Returns the length written,
 * or a negated SPLAX_ERR_* code. */
int splax_profile_report(char *buf, int32_t len);

#ifdef __cplusplus
}
#endif
#endif /* SPLAX_B200_H */
