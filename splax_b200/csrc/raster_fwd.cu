// Forward blend: _rasterize_kernel and _rasterize_depth_kernel
// (splax/_rasterize/_kernels.py:102-205, 277-380).
//
// One 256-thread CTA per (image, 16x16 tile), one pixel per thread. The tile's sorted list is
// walked in batches of 256: each thread gathers one packed 48-byte gaussian record (three
// 16-byte loads from the record array the emission pass wrote) into shared memory, then every
// thread blends the batch front to back from shared memory (broadcast reads). A block vote
// (__syncthreads_count) ends the walk once every pixel's transmittance has saturated.
// Pixel semantics match the reference exactly: a gaussian is skipped when sigma < 0 or
// alpha < 1/255, and the walk stops before the gaussian that would take T to <= 1e-4.
#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

template <bool DEPTH, bool COUNT>
__global__ void __launch_bounds__(kBlockSize)
raster_fwd_kernel(RasterFwdArgs a) {
  unsigned long long evals = 0, contribs = 0;
  __shared__ float4 s_r0[kBlockSize];
  __shared__ float4 s_r1[kBlockSize];
  __shared__ float2 s_r2[kBlockSize];
  const int64_t tile_g = blockIdx.x;
  const int64_t image_id = tile_g / a.num_tiles;
  const int32_t tile_local = static_cast<int32_t>(tile_g % a.num_tiles);
  const int32_t tile_x = tile_local % a.tbx, tile_y = tile_local / a.tbx;
  const int tr = threadIdx.x;
  const int32_t i = tile_y * kBlockWidth + tr / kBlockWidth;
  const int32_t j = tile_x * kBlockWidth + tr % kBlockWidth;
  const float px = static_cast<float>(j) + 0.5f, py = static_cast<float>(i) + 0.5f;
  const bool inside = i < a.img_h && j < a.img_w;
  bool done = !inside;
  const int2 range = reinterpret_cast<const int2*>(a.tile_bins)[tile_g];
  const int32_t range_start = range.x, range_end = range.y;
  const int32_t num_batches = (range_end - range_start + kBlockSize - 1) / kBlockSize;
  float T = 1.0f;
  int32_t cur_idx = 0;
  float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, dep = 0.0f;
  for (int32_t b = 0; b < num_batches; ++b) {
    // block vote doubles as the barrier protecting the previous batch's shared reads
    if (__syncthreads_count(done) >= kBlockSize) break;
    const int32_t batch_start = range_start + b * kBlockSize;
    const int32_t src = batch_start + tr;
    if (src < range_end) {
      const int64_t g = a.gids[src];
      if (g >= 0 && g < a.num_records) {
        const float4* rec = a.records + kRecordFloat4 * g;
        s_r0[tr] = rec[0];
        s_r1[tr] = rec[1];
        const float4 r2 = rec[2];
        s_r2[tr] = make_float2(r2.x, r2.y);
      } else {  // only after a reported emission error: stage a transparent record
        s_r0[tr] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        s_r1[tr] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        s_r2[tr] = make_float2(0.0f, 0.0f);
      }
    }
    __syncthreads();
    const int32_t batch_size = min(kBlockSize, range_end - batch_start);
    if (!done) {
      for (int32_t t = 0; t < batch_size; ++t) {
        const float4 r0 = s_r0[t];
        const float4 r1 = s_r1[t];
        const float dx = r0.x - px, dy = r0.y - py;
        const float sigma = 0.5f * (r0.z * dx * dx + r1.x * dy * dy) + r0.w * dx * dy;
        const float alpha = fminf(kAlphaMax, r1.y * __expf(-sigma));
        if constexpr (COUNT) ++evals;
        if (sigma < 0.0f || alpha < kAlphaThreshold) continue;
        const float next_T = T * (1.0f - alpha);
        if (next_T <= kTransmittanceMin) {
          done = true;
          break;
        }
        const float vis = alpha * T;
        const float2 r2 = s_r2[t];
        c0 += r1.z * vis;
        c1 += r1.w * vis;
        c2 += r2.x * vis;
        if constexpr (DEPTH) dep += r2.y * vis;
        T = next_T;
        cur_idx = batch_start + t;
        if constexpr (COUNT) ++contribs;
      }
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
  if (inside) {
    const float* bg = a.background + 3 * (a.sel_bg ? image_id : 0);
    const int64_t pix = (image_id * a.img_h + i) * static_cast<int64_t>(a.img_w) + j;
    a.final_Ts[pix] = T;
    a.final_idx[pix] = cur_idx;
    a.out_img[3 * pix] = c0 + T * bg[0];
    a.out_img[3 * pix + 1] = c1 + T * bg[1];
    a.out_img[3 * pix + 2] = c2 + T * bg[2];
    if constexpr (DEPTH) a.out_depth[pix] = dep;
  }
}

}  // namespace

void launch_raster_fwd(const RasterFwdArgs& a, cudaStream_t stream) {
  const int64_t blocks = a.num_images * a.num_tiles;
  if (blocks == 0) return;
  const unsigned g = static_cast<unsigned>(blocks);
  if (a.out_depth) {
    if (a.work) raster_fwd_kernel<true, true><<<g, kBlockSize, 0, stream>>>(a);
    else raster_fwd_kernel<true, false><<<g, kBlockSize, 0, stream>>>(a);
  } else {
    if (a.work) raster_fwd_kernel<false, true><<<g, kBlockSize, 0, stream>>>(a);
    else raster_fwd_kernel<false, false><<<g, kBlockSize, 0, stream>>>(a);
  }
}

}  // namespace splax
