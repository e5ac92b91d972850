// Backward blend: _rasterize_bwd_kernel / _rasterize_bwd_agg_kernel and their depth twins
// (splax/_rasterize/_kernels.py:530-794, 935-1209) with _blend_color_vjp / _blend_depth_vjp
// (:1212-1302).
//
// Recompute-style: one 256-thread CTA per (output image, tile), one pixel per thread. The
// walk runs back to front from the block's largest final_idx over batches of 256 records
// staged in shared memory (plus the flat ids that address the gradients). Each pixel rebuilds
// T by dividing out (1 - alpha) and only entries at or below its own final_idx count.
// All lanes of a warp visit the same entry together, so the per-gaussian cotangents (colour 3,
// conic 3, xy 2, opacity 1 [, depth 1]) are summed over the warp with one reduce-scatter
// (~K shuffles for K values) and issued as ONE atomic instruction across K lanes, instead of
// up to K atomics per contributing pixel. Warps with no contributing lane skip the reduction.
#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

template <bool DEPTH, bool COUNT>
__global__ void __launch_bounds__(kBlockSize)
raster_bwd_kernel(RasterBwdArgs a) {
  constexpr int K = DEPTH ? 10 : 9;
  unsigned long long evals = 0, contribs = 0;
  __shared__ float4 s_r0[kBlockSize];
  __shared__ float4 s_r1[kBlockSize];
  __shared__ float2 s_r2[kBlockSize];
  __shared__ int32_t s_id[kBlockSize];
  __shared__ int32_t s_wmax[kBlockSize / 32];

  const int64_t tile_g = blockIdx.x;
  const int64_t image_id = tile_g / a.num_tiles;
  const int32_t tile_local = static_cast<int32_t>(tile_g % a.num_tiles);
  const int64_t geom_image = a.sel_geom ? image_id : 0;
  const int64_t og_base = a.sel_geom ? 0 : image_id * a.n;
  const int2 range = reinterpret_cast<const int2*>(a.tile_bins)[geom_image * a.num_tiles + tile_local];
  const int32_t range_start = range.x, range_end = range.y;
  if (range_end <= range_start) return;

  const int tr = threadIdx.x, lane = tr & 31, warp = tr >> 5;
  const int32_t tile_x = tile_local % a.tbx, tile_y = tile_local / a.tbx;
  const int32_t i = tile_y * kBlockWidth + tr / kBlockWidth;
  const int32_t j = tile_x * kBlockWidth + tr % kBlockWidth;
  const float px = static_cast<float>(j) + 0.5f, py = static_cast<float>(i) + 0.5f;
  const bool inside = i < a.img_h && j < a.img_w;

  int32_t bin_final = range_start - 1;
  float T = 1.0f, t_final = 1.0f;
  float vo0 = 0.0f, vo1 = 0.0f, vo2 = 0.0f, vod = 0.0f, bgdot = 0.0f;
  if (inside) {
    const int64_t fpix = (geom_image * a.img_h + i) * static_cast<int64_t>(a.img_w) + j;
    bin_final = min(a.final_idx[fpix], range_end - 1);
    t_final = a.final_Ts[fpix];
    T = t_final;
    const int64_t vrow = (image_id * a.img_h + i) % a.vout_rows;
    const float* vo = a.v_out_img + 3 * (vrow * a.img_w + j);
    vo0 = vo[0];
    vo1 = vo[1];
    vo2 = vo[2];
    if constexpr (DEPTH) {
      const int64_t drow = (image_id * a.img_h + i) % a.vdepth_rows;
      vod = a.v_out_depth[drow * a.img_w + j];
    }
    const float* bg = a.background + 3 * (a.sel_bg ? image_id : 0);
    bgdot = bg[0] * vo0 + bg[1] * vo1 + bg[2] * vo2;
  }
  float buf0 = 0.0f, buf1 = 0.0f, buf2 = 0.0f, dbuf = 0.0f;

  // gradient slot this lane owns after a reduce-scatter (fixed by the lane id)
  float* my_base = nullptr;
  int my_stride = 0;
  {
    float dummy[K];
#pragma unroll
    for (int k = 0; k < K; ++k) dummy[k] = 0.0f;
    const int c = warp_reduce_scatter<K>(dummy, lane);
    if (c >= 0) {
      if (c < 3) { my_base = a.v_colors + c; my_stride = 3; }
      else if (c < 6) { my_base = a.v_conic + (c - 3); my_stride = 3; }
      else if (c < 8) { my_base = a.v_xy + (c - 6); my_stride = 2; }
      else if (c == 8) { my_base = a.v_opacity; my_stride = 1; }
      else { my_base = a.v_depths; my_stride = 1; }
    }
  }

  // walk starts at the block maximum of final_idx
  const int32_t wmax = __reduce_max_sync(0xffffffffu, bin_final);
  if (lane == 0) s_wmax[warp] = wmax;
  __syncthreads();
  int32_t start_idx = s_wmax[0];
#pragma unroll
  for (int w = 1; w < kBlockSize / 32; ++w) start_idx = max(start_idx, s_wmax[w]);
  const int32_t num_batches = (start_idx - range_start + kBlockSize) / kBlockSize;

  for (int32_t b = 0; b < num_batches; ++b) {
    __syncthreads();  // previous batch's shared reads are complete
    const int32_t batch_end = start_idx - b * kBlockSize;
    const int32_t src = batch_end - tr;
    if (src >= range_start) {
      const int32_t g = a.gids[src];
      if (g >= 0 && g < a.num_records) {
        const float4* rec = a.records + kRecordFloat4 * static_cast<int64_t>(g);
        s_r0[tr] = rec[0];
        s_r1[tr] = rec[1];
        const float4 r2 = rec[2];
        s_r2[tr] = make_float2(r2.x, r2.y);
        s_id[tr] = g;
      } else {  // only after a reported emission error: a transparent record, id 0
        s_r0[tr] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        s_r1[tr] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        s_r2[tr] = make_float2(0.0f, 0.0f);
        s_id[tr] = 0;
      }
    }
    __syncthreads();
    const int32_t batch_size = min(kBlockSize, batch_end - range_start + 1);
    // entries above every pixel of this warp are skipped as a whole
    const int32_t t_begin = max(0, batch_end - wmax);
    for (int32_t t = t_begin; t < batch_size; ++t) {
      const int32_t idx = batch_end - t;
      float v[K];
#pragma unroll
      for (int k = 0; k < K; ++k) v[k] = 0.0f;
      bool contrib = false;
      if (idx <= bin_final) {
        if constexpr (COUNT) ++evals;
        const float4 r0 = s_r0[t];
        const float4 r1 = s_r1[t];
        const float dx = r0.x - px, dy = r0.y - py;
        const float sigma = 0.5f * (r0.z * dx * dx + r1.x * dy * dy) + r0.w * dx * dy;
        if (sigma >= 0.0f) {
          const float vis = __expf(-sigma);
          const float ov = r1.y * vis;
          const float alpha = fminf(kAlphaMax, ov);
          if (alpha >= kAlphaThreshold) {
            contrib = true;
            if constexpr (COUNT) ++contribs;
            const float2 r2 = s_r2[t];
            const float ra = 1.0f / (1.0f - alpha);
            T = T * ra;
            const float fac = alpha * T;
            v[0] = vo0 * fac;
            v[1] = vo1 * fac;
            v[2] = vo2 * fac;
            float v_alpha = (r1.z * T - buf0 * ra) * vo0 + (r1.w * T - buf1 * ra) * vo1 +
                            (r2.x * T - buf2 * ra) * vo2 - t_final * ra * bgdot;
            buf0 += r1.z * fac;
            buf1 += r1.w * fac;
            buf2 += r2.x * fac;
            if constexpr (DEPTH) {
              v_alpha += (r2.y * T - dbuf * ra) * vod;
              dbuf += r2.y * fac;
              v[9] = vod * fac;
            }
            if (ov <= kAlphaMax) {
              const float v_sigma = -ov * v_alpha;
              v[3] = 0.5f * v_sigma * dx * dx;
              v[4] = v_sigma * dx * dy;
              v[5] = 0.5f * v_sigma * dy * dy;
              v[6] = v_sigma * (r0.z * dx + r0.w * dy);
              v[7] = v_sigma * (r0.w * dx + r1.x * dy);
              v[8] = vis * v_alpha;
            }
          }
        }
      }
      if (__ballot_sync(0xffffffffu, contrib) == 0u) continue;
      warp_reduce_scatter<K>(v, lane);
      if (my_base != nullptr && v[0] != 0.0f) {
        const int64_t og = og_base + s_id[t];
        atomicAdd(my_base + og * my_stride, v[0]);
      }
    }
  }
  if constexpr (COUNT) {
    evals = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(evals));
    contribs = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(contribs));
    if (lane == 0) {
      atomicAdd(&a.work[0], evals);
      atomicAdd(&a.work[1], contribs);
    }
  }
}

}  // namespace

void launch_raster_bwd(const RasterBwdArgs& a, cudaStream_t stream) {
  const int64_t blocks = a.B_out * a.num_tiles;
  if (blocks == 0) return;
  const unsigned g = static_cast<unsigned>(blocks);
  if (a.v_out_depth) {
    if (a.work) raster_bwd_kernel<true, true><<<g, kBlockSize, 0, stream>>>(a);
    else raster_bwd_kernel<true, false><<<g, kBlockSize, 0, stream>>>(a);
  } else {
    if (a.work) raster_bwd_kernel<false, true><<<g, kBlockSize, 0, stream>>>(a);
    else raster_bwd_kernel<false, false><<<g, kBlockSize, 0, stream>>>(a);
  }
}

}  // namespace splax
