// Kernel argument blocks and launchers shared between the .cu files of libsplax_b200.
// Host-only interface: the C-ABI in capi.cu fills these from the caller's pointers and sizes.
#pragma once

#include <cstdint>
#include <cstdio>
#include <string>
#include <cuda_runtime.h>

namespace splax {

// Zero-filled device spans (4-byte aligned, whole 4-byte words), cleared by one launch_pdl
// kernel instead of one cudaMemsetAsync each, so the launch chain stays programmatic.
struct ClearSpan {
  void* p;
  size_t bytes;
};
constexpr int kClearMaxSpans = 6;
void launch_clear(const ClearSpan* spans, int count, cudaStream_t stream);

// Launch with programmatic stream serialization: the kernel (which begins with pdl_enter) may
// be scheduled while its stream predecessor finishes. Errors surface through cudaGetLastError
// like a <<<>>> launch.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  (void)cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

struct ProjectArgs {
  const float* means;
  const float* scales;
  const float* quats;  // xyzw
  const float* viewmat;
  const float* opacities;
  const float* transforms;
  const int32_t* transform_ids;
  int64_t n, total;
  int32_t num_transforms;
  bool has_transforms, sel_means, sel_scales, sel_quats, sel_view, sel_opac, sel_transforms;
  int32_t img_h, img_w;
  float fx, fy, cx, cy, glob_scale, clip_thresh;
  float* xys;
  float* depths;
  int32_t* radii;
  float* conics;
  int32_t* num_tiles_hit;
  int32_t* cum_tiles_hit;
  // antialiased mode (optional): rho = sqrt(clip(1 - eps (a + c) + eps^2 (a c - b^2), 0, 1))
  // of the dilated conic per pair, 1 when culled; nullptr skips it
  float* rho = nullptr;
  float aa_eps = 0.0f, aa_eps2 = 0.0f;
  bool quats_wxyz = false;  // quaternions stored scalar-first
};

struct ProjectBwdArgs {
  const float* means;
  const float* scales;
  const float* quats;
  const float* viewmat;
  const int32_t* radii;
  const float* conics;
  const float* v_xy;     // nullptr: zero cotangent
  const float* v_depth;  // nullptr: zero cotangent
  const float* v_conic;
  const float* transforms;
  const int32_t* transform_ids;
  int64_t n, B;
  int32_t num_transforms;
  bool has_transforms, sel_means, sel_scales, sel_quats, sel_view, sel_radii, sel_conics,
      sel_vxy, sel_vdepth, sel_vconic, sel_transforms;
  float fx, fy, glob_scale;
  float* v_mean3d;
  float* v_scale;
  float* v_quat;
  float* v_viewmat;     // (B, 4, 4), zeroed by the caller
  float* v_transforms;  // (B, K, 4, 4), zeroed by the caller
  // antialiased mode (optional): cotangent of the forward's rho, chained into the conic's
  const float* v_rho = nullptr;
  bool sel_vrho = false;
  float aa_eps = 0.0f, aa_eps2 = 0.0f;
  bool quats_wxyz = false;  // quaternions (and v_quat) stored scalar-first
  // v_mean3d / v_scale / v_quat hold n rows summed over the B images (shared operands)
  bool fold_batch = false;
};

// Per-gaussian record staged by the blend kernels: 3 x float4 =
// (x, y, qa, qb), (qc, opacity, r, g), (b, depth, log2 opacity, 0), with the conic pre-scaled
// for a base-2 exponent, (qa, qb, qc) = -log2(e)/2 * (a, 2b, c), and log2(opacity) added to the
// exponent so that alpha = 2^p; the last float pads the record to 16-byte loads.
constexpr int kRecordFloat4 = 3;

struct EmitArgs {
  const int32_t* perm;     // pairs in (image, depth key) order
  const int32_t* dtotal = nullptr;  // device-side number of sorted pairs (<= total), or nullptr
  const int32_t* offsets;  // exclusive scan of their tile counts in that order
  const int32_t* counts;   // tile count per pair (flat order)
  const float4* walk;      // walk record per pair (flat order)
  int64_t total;
  int64_t count;  // intersections (cum[total-1]); emission never writes past it
  int32_t tile_n_bits, tbx, tby;
  uint32_t* keys;  // (image | tile) bin keys
  int32_t* vals;
  unsigned* err;
};

struct PairKeyArgs {
  const float* depths;
  const int32_t* radii;
  const int32_t* depth_mm;  // ordered-int per-image [min, max] of visible depths
  int64_t n, total;
  bool packed;         // quantised depth (32-bit reference keys) or float bits (64-bit)
  int32_t depth_bits;  // packed: the reference's depth field width
  int32_t key_shift;   // bits below the image id in the pair key
  unsigned* err;
  // per-pair records (flat order); walk == nullptr skips them
  const float* xys;
  const float* conics;
  const int32_t* cum;
  const float* map_opacities;
  int64_t map_opac_rows;
  const float* opacities;
  int64_t opac_rows;
  const float* colors;
  int64_t color_rows;
  int32_t* counts;
  float4* walk;     // (x, y, a, b), (c, iso level, image id bits, count bits)
  float4* records;  // blend records, nullptr without colours
};

void launch_project_fwd(const ProjectArgs& a, unsigned long long* status, int* ticket,
                        unsigned* err, cudaStream_t stream);
// The projection's fused scan covers kProjScanTile pairs per CTA and keeps one look-back word
// per such tile.
constexpr int64_t kProjScanTile = 1024;
int64_t project_scan_tiles(int64_t total);
void launch_project_bwd(const ProjectBwdArgs& a, cudaStream_t stream);

// sort.cu
void launch_depth_minmax(const float* depths, const int32_t* radii, int64_t total, int64_t n,
                         int32_t B, int32_t* depth_mm, cudaStream_t stream);
void launch_depth_span(const int32_t* depth_mm, int32_t B, unsigned* span_out,
                       cudaStream_t stream);
void launch_pair_keys(const PairKeyArgs& a, bool key64, void* keys, int32_t* vals,
                      cudaStream_t stream);
int64_t sorted_offsets_tiles(int64_t total);
void launch_sorted_offsets(const int32_t* perm, const int32_t* counts, int64_t total,
                           const int32_t* dtotal, int32_t* offsets, unsigned long long* status,
                           int* ticket, unsigned* err, cudaStream_t stream);
void launch_emit(const EmitArgs& a, cudaStream_t stream);
void launch_reference_keys(const uint32_t* bin_keys, const int32_t* gids, int64_t count,
                           const PairKeyArgs& a, int64_t* out, cudaStream_t stream);
// Onesweep radix sort of (key, value) pairs over `bits` low key bits, ping-ponging between
// the two buffers; returns the index (0 or 1) of the buffer holding the result.
struct SortScratch {
  void* keys[2];
  int32_t* vals[2];
  uint32_t* hist;                 // [passes][256] counts, then [passes][256] offsets
  unsigned long long* status;     // look-back words, status_words entries
  int64_t status_words;
  // drop all-ones keys (the first pass writes only the others) and write how many keys were
  // sorted to vcount, which the later passes read
  bool filter_sentinel = false;
  int32_t* vcount = nullptr;
  int* tile_counters;             // one per pass
  unsigned* err;
};
int sort_tile_items(bool key64);
// Radix passes a sort of `bits` significant bits takes (8- or 9-bit digits; look-back words per
// tile: 2^digit bits, at most kRadixMaxDigits).
int radix_passes(int bits);
constexpr int kRadixMaxDigits = 512;
int radix_sort_pairs(const SortScratch& s, bool key64, int64_t count, int bits,
                     cudaStream_t stream);
void launch_tile_bins(const uint32_t* keys, int64_t count, int32_t tile_n_bits,
                      int32_t num_tiles, int64_t num_bins, int32_t* tile_bins, unsigned* err,
                      cudaStream_t stream);

// raster_fwd.cu
struct RasterFwdArgs {
  int32_t img_h, img_w, tbx, num_tiles;
  int64_t num_images;
  const int32_t* tile_bins;  // int2 per bin
  const int32_t* gids;
  const float4* records;
  int64_t num_records;  // flat ids outside [0, num_records) are staged as transparent
  const float* background;
  bool sel_bg;
  float* final_Ts;
  int32_t* final_idx;
  float* out_img;
  float* out_depth;  // nullptr for the plain blend
  unsigned long long* work;  // optional: [0] evaluations, [1] contributions
};
void launch_raster_fwd(const RasterFwdArgs& a, cudaStream_t stream);

// raster_bwd.cu
struct RasterBwdArgs {
  int32_t img_h, img_w, tbx, num_tiles;
  int64_t n, B_out;
  bool sel_geom, sel_bg;
  int64_t vout_rows, vdepth_rows;
  const int32_t* tile_bins;
  const int32_t* gids;
  const float4* records;
  int64_t num_records;
  const float* background;
  const float* final_Ts;
  const int32_t* final_idx;
  const float* v_out_img;
  const float* v_out_depth;  // nullptr for the plain blend
  float* v_colors;
  float* v_opacity;
  float* v_xy;
  float* v_conic;
  float* v_depths;
  // v_colors / v_opacity hold n rows, each summed over the images (shared operands)
  bool fold_colors = false, fold_opacity = false;
  unsigned long long* work;  // optional: [0] evaluations, [1] contributions
};
void launch_raster_bwd(const RasterBwdArgs& a, cudaStream_t stream);

// capi.cu: set the calling thread's splax_last_error() message and return `code`
int record_error(int code, const char* msg);

// Fused MSE loss (loss.cu). `partials` holds `blocks` doubles; `done` is a zeroed counter the
// kernel leaves zeroed.
int mse_loss_blocks();
void launch_mse_loss(const float* img, const float* tgt, int64_t count, double inv_denom,
                     double* partials, unsigned* done, float* loss, int blocks,
                     cudaStream_t stream);
void launch_mse_loss_bwd(const float* img, const float* tgt, int64_t count, float scale,
                         const float* v_loss, float* grad, int blocks, cudaStream_t stream);

// Fused L1 + D-SSIM loss (ssim.cu). The 11 window weights are set once per device.
void ssim_set_window(const float* w11);
int64_t l1_dssim_partials(int32_t B, int32_t H, int32_t W);
void launch_l1_dssim(const float* img, const float* tgt, int32_t B, int32_t H, int32_t W,
                     double l1_scale, double ssim_scale, double ssim_const, double2* partials,
                     float* loss, cudaStream_t stream);
void launch_l1_dssim_bwd(const float* img, const float* tgt, int32_t B, int32_t H, int32_t W,
                         float l1_scale, float ssim_grad_scale, const float* v_loss, float* grad,
                         cudaStream_t stream);
// The loss and its gradient for a unit cotangent in one pass (the backward kernel, which also
// sums the map entries and L1 it owns); partials: l1_dssim_partials_max entries.
int64_t l1_dssim_partials_max(int32_t B, int32_t H, int32_t W);
void launch_l1_dssim_and_grad(const float* img, const float* tgt, int32_t B, int32_t H,
                              int32_t W, double l1_scale, double ssim_scale, double ssim_const,
                              float l1_grad_scale, float ssim_grad_scale, double2* partials,
                              float* loss, float* grad, cudaStream_t stream);

// Fused multi-array Adam (optim.cu): up to kAdamMaxSegs parameter arrays per launch.
constexpr int kAdamMaxSegs = 8;
struct AdamSeg {
  float* p;
  const float* g;
  float* m;
  float* v;
  int64_t n;
  float lr;
};
struct AdamSegs {
  AdamSeg seg[kAdamMaxSegs];
};
void launch_adam(const AdamSegs& s, int32_t count, float b1, float b2, float bc1, float bc2,
                 float eps, cudaStream_t stream);

// 3DGS .ply loading (ply.cu): byte offsets of x y z, scale_0..2, rot_0..3, f_dc_0..2, opacity
// in a vertex record of `stride` bytes.
struct PlyLayout {
  int32_t off[14];
  int64_t stride;
  bool aligned;  // every needed offset and the stride are multiples of 4
};
// collective.cu: NVLS gradient all-reduce. flags: host array of `world` device pointers, each
// rank's u64[world] flag array (all zero before the first epoch; epochs increase per call).
int launch_nvls_barrier(unsigned long long* const* flags, int rank, int world,
                        unsigned long long epoch, unsigned* err, cudaStream_t stream);
// In-place sum over the ranks of n floats at the multicast address (16-byte aligned); does
// nothing once *err (this rank's error word) is nonzero.
int launch_nvls_allreduce(float* multicast, int64_t n, int rank, int world, const unsigned* err,
                          cudaStream_t stream);
// Fused exchange and Adam update of a flat parameter buffer split in up to kAdamMaxSegs groups
// (group k holds the elements below end[k], learning rate lr[k]).
struct NvlsAdamGroups {
  int64_t end[kAdamMaxSegs];
  float lr[kAdamMaxSegs];
  int32_t count;
};
// Moments this rank holds (floats): 4 x its shard's vectors, plus the n % 4 tail on the last rank.
int64_t nvls_adam_shard_len(int64_t n, int rank, int world);
int launch_nvls_adam(const float* grad_mc, float* param_mc, const float* param_local,
                     float* m_shard, float* v_shard, int64_t n, int rank, int world,
                     const NvlsAdamGroups& gr, float b1, float b2, float bc1, float bc2, float eps,
                     const unsigned* err, cudaStream_t stream);

int ply_parse_header(FILE* f, PlyLayout* L, int64_t* count, int64_t* body_offset,
                     std::string* why);
void launch_ply_decode(const unsigned char* body, int64_t count, const PlyLayout& L,
                       int64_t first, float* means, float* scales, float* quats, float* colors,
                       float* opacities, cudaStream_t stream);

}  // namespace splax
