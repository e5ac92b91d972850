// Forward blend: _rasterize_kernel and _rasterize_depth_kernel
// (splax/_rasterize/_kernels.py:102-205, 277-380).
//
// One 64-thread CTA per (image, 16x16 tile); each warp owns a 16x8 block of the tile and each
// thread four vertically adjacent pixels, so every shared-memory record read and the x-terms of
// the Gaussian exponent serve four evaluations; the exponents are computed as two pairs with
// packed fp32x2 instructions, the blend step per pixel with one branch for "skip" (a finished
// pixel, or the reference's sigma / alpha tests) and one for termination. The tile's sorted list
// is walked in batches of 256: the CTA gathers the packed 48-byte records (three 16-byte loads
// each, written by the emission pass) into shared memory, then blends the batch front to back
// from shared memory with broadcast reads, two records per loop trip. Records carry the conic
// pre-scaled by -log2(e)/2 and log2(opacity), which is added to the x-term once per record, so
// p = log2(alpha) is a quadratic form evaluated with FMAs and alpha one ex2 (no multiply).
// A block vote (__syncthreads_count) ends the walk once every pixel has saturated.
//
// Pixel semantics are the reference's: a gaussian is skipped when sigma < 0 (p > log2 opacity)
// or alpha < 1/255, and the walk stops before the gaussian that would take T to <= 1e-4. The
// transmittance update T (1 - alpha) is one FMA, T - alpha T rounded once, where the reference
// rounds 1 - alpha and the product separately: within an ulp of it per step.
//
// The alpha clamp min(0.999, 2^p) can only act on a gaussian whose opacity is close to 0.999,
// since p <= log2(opacity) for every gaussian that is not skipped. Each staged batch
// notes whether any of its records has an opacity above kClampFreeOpacity; batches without one
// (all of them for most scenes) run a loop without the clamp, whose results are identical.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {
// the record loop unrolled by two: the next record's exponents overlap this one's blend
// (1.84 -> 1.76 ms; by four: 1.79)
constexpr int kFwdUnroll = 2;
// Below this opacity alpha = ex2.approx(p) stays under 0.999 for every p <= log2(opacity) (the
// approximation's relative error, about 2^-22, and the rounding of p leave it within 1.001 of
// the opacity), so min(0.999, alpha) == alpha exactly.
constexpr float kClampFreeOpacity = 0.998f;


struct PixelState {
  float T = 1.0f, c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, dep = 0.0f;
  int32_t cur_idx = 0;
  bool done;
};

// The reference blend step (splax/_rasterize/_kernels.py:185-197) for one pixel.
template <bool DEPTH, bool COUNT, bool CLAMP>
__device__ __forceinline__ void blend_one(PixelState& s, float p, float lo, float r, float g,
                                          float b, float depth, int32_t idx, int& ndone,
                                          unsigned long long& evals,
                                          unsigned long long& contribs) {
  // the skip tests of a done pixel and of the reference's sigma / alpha tests share one branch
  if constexpr (COUNT) evals += s.done ? 0 : 1;
  // p carries log2(opacity): alpha = 2^p, and the exponent itself is p - lo
  const float ov = ex2_approx(p);
  // min(0.999, ov) < 1/255 exactly when ov < 1/255
  if (s.done || p > lo || ov < kAlphaThreshold) return;
  const float alpha = CLAMP ? fminf(kAlphaMax, ov) : ov;
  const float next_T = fmaf(-alpha, s.T, s.T);  // T (1 - alpha), rounded once
  if (next_T <= kTransmittanceMin) {
    s.done = true;
    ++ndone;
    return;
  }
  const float vis = alpha * s.T;
  s.c0 += r * vis;
  s.c1 += g * vis;
  s.c2 += b * vis;
  if constexpr (DEPTH) s.dep += depth * vis;
  s.T = next_T;
  s.cur_idx = idx;
  if constexpr (COUNT) ++contribs;
}

// Four vertically adjacent pixels per thread (exponents computed as two packed pairs); a warp
// owns a 16x8 block of the tile and the 64-thread CTA the whole tile.
constexpr int kPixels = 4;
constexpr int kPairs = kPixels / 2;

template <bool DEPTH, bool COUNT>
__global__ void __launch_bounds__(kBlockSize / kPixels)
raster_fwd_kernel(RasterFwdArgs a) {
  pdl_enter();
  constexpr int kFwdThreads = kBlockSize / kPixels;
  unsigned long long evals = 0, contribs = 0;
  __shared__ float4 s_r0[kBlockSize];
  __shared__ float4 s_r1[kBlockSize];
  // (b, log2 opacity), or (b, depth, log2 opacity, 0) with depth
  __shared__ std::conditional_t<DEPTH, float4, float2> s_r2[kBlockSize];
  const int64_t tile_g = blockIdx.x;
  const int64_t image_id = tile_g / a.num_tiles;
  const int32_t tile_local = static_cast<int32_t>(tile_g % a.num_tiles);
  const int32_t tile_x = tile_local % a.tbx, tile_y = tile_local / a.tbx;
  const int tr = threadIdx.x, lane = tr & 31, warp = tr >> 5;
  const int32_t j = tile_x * kBlockWidth + (lane & 15);
  const int32_t i0 = tile_y * kBlockWidth + 2 * kPixels * warp + kPixels * (lane >> 4);
  const float px = static_cast<float>(j) + 0.5f;
  const float py0 = static_cast<float>(i0) + 0.5f;
  PixelState st[kPixels];
  int ndone = 0;  // pixels of this thread that are done (outside the image or saturated)
#pragma unroll
  for (int k = 0; k < kPixels; ++k) {
    st[k].done = !(i0 + k < a.img_h && j < a.img_w);
    ndone += st[k].done ? 1 : 0;
  }
  const int2 range = reinterpret_cast<const int2*>(a.tile_bins)[tile_g];
  const int32_t range_start = range.x, range_end = range.y;
  const int32_t num_batches = (range_end - range_start + kBlockSize - 1) / kBlockSize;
  for (int32_t bt = 0; bt < num_batches; ++bt) {
    // block vote doubles as the barrier protecting the previous batch's shared reads
    if (__syncthreads_count(ndone == kPixels) >= kFwdThreads) break;
    const int32_t batch_start = range_start + bt * kBlockSize;
    bool high_opacity = false;
#pragma unroll
    for (int h = 0; h < kBlockSize / kFwdThreads; ++h) {
      const int slot = tr + h * kFwdThreads;
      const int32_t src = batch_start + slot;
      if (src < range_end) {
        const int64_t g = a.gids[src];
        if (g >= 0 && g < a.num_records) {
          const float4* rec = a.records + kRecordFloat4 * g;
          s_r0[slot] = rec[0];
          const float4 r1 = rec[1];
          s_r1[slot] = r1;
          high_opacity |= r1.y > kClampFreeOpacity;
          const float4 r2 = rec[2];
          if constexpr (DEPTH) s_r2[slot] = r2;
          else s_r2[slot] = make_float2(r2.x, r2.z);
        } else {  // only after a reported emission error: stage a transparent record
          s_r0[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          s_r1[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if constexpr (DEPTH) s_r2[slot] = make_float4(0.0f, 0.0f, neg_inf(), 0.0f);
          else s_r2[slot] = make_float2(0.0f, neg_inf());
        }
      }
    }
    // the barrier publishing the batch also tells every thread whether it needs the clamp
    const bool clamp = __syncthreads_or(high_opacity) != 0;
    const int32_t batch_size = min(kBlockSize, range_end - batch_start);
    auto blend_batch = [&](auto clamp_tag) {
      constexpr bool kClamp = decltype(clamp_tag)::value;
#pragma unroll kFwdUnroll
      for (int32_t t = 0; t < batch_size; ++t) {
        const float4 r0 = s_r0[t];  // x, y, qa, qb  (q = -log2(e)/2 * (a, 2b, c))
        const float4 r1 = s_r1[t];  // qc, opacity, r, g
        const auto r2 = s_r2[t];
        float b, depth, lo;
        if constexpr (DEPTH) { b = r2.x; depth = r2.y; lo = r2.z; }
        else { b = r2.x; depth = 0.0f; lo = r2.y; }
        const float dx = r0.x - px;
        const float dy0 = r0.y - py0;
        // the x-term carries log2(opacity): one explicit FMA, as the backward computes it
        const float2 qxx = splat2(fmaf(r0.z * dx, dx, lo)), qbx = splat2(r0.w * dx),
                     qc = splat2(r1.x);
        const int32_t idx = batch_start + t;
#pragma unroll
        for (int q = 0; q < kPairs; ++q) {
          // the exponents of a pixel pair in packed form, then the branchy per-pixel step
          const float2 dy = add2(splat2(dy0), make_float2(-2.0f * q, -2.0f * q - 1.0f));
          const float2 p = fma2(fma2(qc, dy, qbx), dy, qxx);
          blend_one<DEPTH, COUNT, kClamp>(st[2 * q], p.x, lo, r1.z, r1.w, b, depth, idx, ndone,
                                          evals, contribs);
          blend_one<DEPTH, COUNT, kClamp>(st[2 * q + 1], p.y, lo, r1.z, r1.w, b, depth, idx,
                                          ndone, evals, contribs);
        }
        // tested once per pair of records (the loop is unrolled by two): 1.708 -> 1.685 ms
        // per config-2 step together with the single-rounding transmittance update
        if ((t & 1) && ndone == kPixels) break;
      }
    };
    if (ndone < kPixels) {
      if (clamp) blend_batch(std::true_type{});
      else blend_batch(std::false_type{});
    }
  }
  if constexpr (COUNT) {
    evals = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(evals));
    contribs = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(contribs));
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&a.work[0], evals);
      atomicAdd(&a.work[1], contribs);
    }
  }
  const float* bg = a.background + 3 * (a.sel_bg ? image_id : 0);
  const float bg0 = bg[0], bg1 = bg[1], bg2 = bg[2];
#pragma unroll
  for (int k = 0; k < kPixels; ++k) {
    const PixelState& s = st[k];
    const int32_t i = i0 + k;
    if (!(i < a.img_h && j < a.img_w)) continue;
    const int64_t pix = (image_id * a.img_h + i) * static_cast<int64_t>(a.img_w) + j;
    a.final_Ts[pix] = s.T;
    a.final_idx[pix] = s.cur_idx;
    a.out_img[3 * pix] = s.c0 + s.T * bg0;
    a.out_img[3 * pix + 1] = s.c1 + s.T * bg1;
    a.out_img[3 * pix + 2] = s.c2 + s.T * bg2;
    if constexpr (DEPTH) a.out_depth[pix] = s.dep;
  }
}

void launch_fwd(const RasterFwdArgs& a, unsigned g, cudaStream_t stream) {
  constexpr int nt = kBlockSize / kPixels;
  if (a.out_depth) {
    if (a.work) launch_pdl(raster_fwd_kernel<true, true>, g, nt, 0, stream, a);
    else launch_pdl(raster_fwd_kernel<true, false>, g, nt, 0, stream, a);
  } else {
    if (a.work) launch_pdl(raster_fwd_kernel<false, true>, g, nt, 0, stream, a);
    else launch_pdl(raster_fwd_kernel<false, false>, g, nt, 0, stream, a);
  }
}

}  // namespace

void launch_raster_fwd(const RasterFwdArgs& a, cudaStream_t stream) {
  const int64_t blocks = a.num_images * a.num_tiles;
  if (blocks == 0) return;
  const unsigned g = static_cast<unsigned>(blocks);
  launch_fwd(a, g, stream);
}

}  // namespace splax
