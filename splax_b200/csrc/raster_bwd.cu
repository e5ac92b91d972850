// Backward blend: _rasterize_bwd_kernel / _rasterize_bwd_agg_kernel and their depth twins
// (splax/_rasterize/_kernels.py:530-794, 935-1209) with _blend_color_vjp / _blend_depth_vjp
// (:1212-1302).
//
// Recompute-style: one 64-thread CTA per (output image, tile); each warp owns a 16x8 block and
// each thread four vertically adjacent pixels. A warp skips every gaussian whose alpha >= 1/255
// ellipse misses its block (those evaluations are all rejected). The walk runs back to front from the block's largest
// final_idx over batches of 256 records staged in shared memory (plus the flat ids that
// address the gradients). Each pixel rebuilds T by dividing out (1 - alpha), and only entries
// at or below its own final_idx count. All lanes of a warp visit the same entry together, so
// each thread first adds its two pixels' cotangents, then the warp sums the 9 (10 with depth)
// per-gaussian values with one reduce-scatter (~K shuffles instead of 5K) and issues ONE atomic
// instruction across K lanes. Warps where no pixel contributes skip the reduction.
//
// The staged conic is pre-scaled (q = -log2(e)/2 * (a, 2b, c)), so the exponent is one ex2;
// the xy cotangent rescales by -ln 2 to recover the conic.
#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

constexpr float kLn2 = 0.693147180559945f;

struct BwdPixel {
  int32_t bin_final;
  float T, vo0, vo1, vo2, vod;
  float tb;            // t_final * (background . v_out): the background's share of v_alpha
  float bufdot = 0.0f; // (colour, depth) accumulated behind this gaussian, dotted with v_out
};

// Accumulators of one thread for the current gaussian, over its two pixels:
// [0..2] colour, [3] sum v_sigma, [4] sum v_sigma dy, [5] sum v_sigma dy^2, [6] opacity,
// [7] depth. The xy and conic cotangents are formed from these once per thread.
//
// _blend_color_vjp (splax/_rasterize/_kernels.py:1212-1254) restated with the colour buffer
// kept as its dot product with v_out: v_alpha = T (c . v_out) - ra (buf . v_out + t_final
// bg . v_out), and buf . v_out grows by (c . v_out) fac.
template <bool DEPTH>
__device__ __forceinline__ bool vjp_one(BwdPixel& s, int32_t idx, float p, float dy, float opac,
                                        float r, float g, float b, float depth, float* acc) {
  if (idx > s.bin_final || p > 0.0f) return false;
  const float vis = ex2_approx(p);
  const float ov = opac * vis;
  const float alpha = fminf(kAlphaMax, ov);
  if (alpha < kAlphaThreshold) return false;
  const float ra = __fdividef(1.0f, 1.0f - alpha);
  s.T = s.T * ra;
  const float fac = alpha * s.T;
  acc[0] += s.vo0 * fac;
  acc[1] += s.vo1 * fac;
  acc[2] += s.vo2 * fac;
  float cv = r * s.vo0 + g * s.vo1 + b * s.vo2;
  if constexpr (DEPTH) {
    cv += depth * s.vod;
    acc[7] += s.vod * fac;
  }
  const float v_alpha = s.T * cv - ra * (s.bufdot + s.tb);
  s.bufdot += cv * fac;
  // where the 0.999 clamp is active alpha is constant: no sigma or opacity cotangent
  const bool live = ov <= kAlphaMax;
  const float vs = live ? -ov * v_alpha : 0.0f;
  acc[6] += live ? vis * v_alpha : 0.0f;
  acc[3] += vs;
  const float vsy = vs * dy;
  acc[4] += vsy;
  acc[5] += vsy * dy;
  return true;
}

// PIX vertically adjacent pixels per thread; a warp owns a 16 x (2 PIX) block of the tile and
// the CTA (256 / PIX threads) the whole tile. Four pixels per thread amortise the per-gaussian
// warp reduction over 128 pixels.
constexpr int kPixels = 4;

template <bool DEPTH, bool COUNT, int PIX>
__global__ void __launch_bounds__(kBlockSize / PIX)
raster_bwd_kernel(RasterBwdArgs a) {
  constexpr int kBwdThreads = kBlockSize / PIX;
  constexpr int K = DEPTH ? 10 : 9;
  unsigned long long evals = 0, contribs = 0;
  unsigned steps = 0, steps_uncull = 0, steps_active = 0;  // warp steps (COUNT builds only)
  __shared__ float4 s_r0[kBlockSize];
  __shared__ float4 s_r1[kBlockSize];
  __shared__ float4 s_r2[kBlockSize];
  __shared__ int32_t s_id[kBlockSize];
  __shared__ int32_t s_wmax[kBwdThreads / 32];

  const int64_t tile_g = blockIdx.x;
  const int64_t image_id = tile_g / a.num_tiles;
  const int32_t tile_local = static_cast<int32_t>(tile_g % a.num_tiles);
  const int64_t geom_image = a.sel_geom ? image_id : 0;
  const int64_t og_base = a.sel_geom ? 0 : image_id * a.n;
  const int2 range =
      reinterpret_cast<const int2*>(a.tile_bins)[geom_image * a.num_tiles + tile_local];
  const int32_t range_start = range.x, range_end = range.y;
  if (range_end <= range_start) return;

  const int tr = threadIdx.x, lane = tr & 31, warp = tr >> 5;
  const int32_t tile_x = tile_local % a.tbx, tile_y = tile_local / a.tbx;
  const int32_t j = tile_x * kBlockWidth + (lane & 15);
  const int32_t i0 = tile_y * kBlockWidth + 2 * PIX * warp + PIX * (lane >> 4);
  const float px = static_cast<float>(j) + 0.5f;
  const float py0 = static_cast<float>(i0) + 0.5f;
  // centre of the warp's block of pixel centres (half-extents 7.5 and PIX - 0.5)
  const float wcx = static_cast<float>(tile_x * kBlockWidth) + 8.0f;
  const float wcy = static_cast<float>(tile_y * kBlockWidth + 2 * PIX * warp + PIX);
  constexpr float kHalfY = PIX - 0.5f;

  BwdPixel px_s[PIX];
  const float* bg = a.background + 3 * (a.sel_bg ? image_id : 0);
#pragma unroll
  for (int k = 0; k < PIX; ++k) {
    BwdPixel& s = px_s[k];
    const int32_t i = i0 + k;
    s.bin_final = range_start - 1;
    s.T = 1.0f;
    s.vo0 = s.vo1 = s.vo2 = s.vod = s.tb = 0.0f;
    if (i < a.img_h && j < a.img_w) {
      const int64_t fpix = (geom_image * a.img_h + i) * static_cast<int64_t>(a.img_w) + j;
      s.bin_final = min(a.final_idx[fpix], range_end - 1);
      const float t_final = a.final_Ts[fpix];
      s.T = t_final;
      const int64_t vrow = (image_id * a.img_h + i) % a.vout_rows;
      const float* vo = a.v_out_img + 3 * (vrow * a.img_w + j);
      s.vo0 = vo[0];
      s.vo1 = vo[1];
      s.vo2 = vo[2];
      if constexpr (DEPTH) {
        const int64_t drow = (image_id * a.img_h + i) % a.vdepth_rows;
        s.vod = a.v_out_depth[drow * a.img_w + j];
      }
      s.tb = t_final * (bg[0] * s.vo0 + bg[1] * s.vo1 + bg[2] * s.vo2);
    }
  }

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
  int32_t tmax = px_s[0].bin_final;
#pragma unroll
  for (int k = 1; k < PIX; ++k) tmax = max(tmax, px_s[k].bin_final);
  const int32_t wmax = __reduce_max_sync(0xffffffffu, tmax);
  if (lane == 0) s_wmax[warp] = wmax;
  __syncthreads();
  int32_t start_idx = s_wmax[0];
#pragma unroll
  for (int w = 1; w < kBwdThreads / 32; ++w) start_idx = max(start_idx, s_wmax[w]);
  const int32_t num_batches = (start_idx - range_start + kBlockSize) / kBlockSize;

  for (int32_t b = 0; b < num_batches; ++b) {
    __syncthreads();  // previous batch's shared reads are complete
    const int32_t batch_end = start_idx - b * kBlockSize;
#pragma unroll
    for (int h = 0; h < kBlockSize / kBwdThreads; ++h) {
      const int slot = tr + h * kBwdThreads;
      const int32_t src = batch_end - slot;
      if (src >= range_start) {
        const int32_t g = a.gids[src];
        if (g >= 0 && g < a.num_records) {
          const float4* rec = a.records + kRecordFloat4 * static_cast<int64_t>(g);
          s_r0[slot] = rec[0];
          s_r1[slot] = rec[1];
          s_r2[slot] = rec[2];
          s_id[slot] = g;
        } else {  // only after a reported emission error: a transparent record, id 0
          s_r0[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          s_r1[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          s_r2[slot] = make_float4(0.0f, 0.0f, -1.0e30f, -1.0e30f);
          s_id[slot] = 0;
        }
      }
    }
    __syncthreads();
    const int32_t batch_size = min(kBlockSize, batch_end - range_start + 1);
    // entries above every pixel of this warp are skipped as a whole
    const int32_t t_begin = max(0, batch_end - wmax);
    for (int32_t t = t_begin; t < batch_size; ++t) {
      const int32_t idx = batch_end - t;
      const float4 r0 = s_r0[t];
      const float4 r2 = s_r2[t];
      if constexpr (COUNT) {
#pragma unroll
        for (int k = 0; k < PIX; ++k) evals += idx <= px_s[k].bin_final;
        ++steps;
      }
      if (fabsf(r0.x - wcx) > r2.z + 7.5f || fabsf(r0.y - wcy) > r2.w + kHalfY) continue;
      if constexpr (COUNT) ++steps_uncull;
      const float4 r1 = s_r1[t];
      const float dx = r0.x - px;
      const float dy0 = r0.y - py0;
      const float qxx = r0.z * dx * dx, qbx = r0.w * dx;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
      bool any = false;
#pragma unroll
      for (int k = 0; k < PIX; ++k) {
        const float dy = dy0 - static_cast<float>(k);
        const float p = fmaf(fmaf(r1.x, dy, qbx), dy, qxx);
        const bool c = vjp_one<DEPTH>(px_s[k], idx, p, dy, r1.y, r1.z, r1.w, r2.x, r2.y, acc);
        if constexpr (COUNT) contribs += c;
        any |= c;
      }
      if (__ballot_sync(0xffffffffu, any) == 0u) continue;
      if constexpr (COUNT) ++steps_active;
      // per-thread cotangents: sum_px v_sigma (dx, dy) and the second moments give the conic
      // and xy terms; (a, b, c) = -ln2 (2 qa, qb, 2 qc) recovers the unscaled conic
      const float sx = acc[3] * dx, sy = acc[4];
      const float a2 = -2.0f * kLn2 * r0.z, bq = -kLn2 * r0.w, c2 = -2.0f * kLn2 * r1.x;
      float v[K];
      v[0] = acc[0];
      v[1] = acc[1];
      v[2] = acc[2];
      v[3] = 0.5f * sx * dx;
      v[4] = sy * dx;
      v[5] = 0.5f * acc[5];
      v[6] = fmaf(a2, sx, bq * sy);
      v[7] = fmaf(bq, sx, c2 * sy);
      v[8] = acc[6];
      if constexpr (DEPTH) v[9] = acc[7];
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
      atomicAdd(&a.work[2], static_cast<unsigned long long>(steps));
      atomicAdd(&a.work[3], static_cast<unsigned long long>(steps_uncull));
      atomicAdd(&a.work[4], static_cast<unsigned long long>(steps_active));
    }
  }
}

template <int PIX>
void launch_bwd(const RasterBwdArgs& a, unsigned g, cudaStream_t stream) {
  constexpr int nt = kBlockSize / PIX;
  if (a.v_out_depth) {
    if (a.work) raster_bwd_kernel<true, true, PIX><<<g, nt, 0, stream>>>(a);
    else raster_bwd_kernel<true, false, PIX><<<g, nt, 0, stream>>>(a);
  } else {
    if (a.work) raster_bwd_kernel<false, true, PIX><<<g, nt, 0, stream>>>(a);
    else raster_bwd_kernel<false, false, PIX><<<g, nt, 0, stream>>>(a);
  }
}

}  // namespace

void launch_raster_bwd(const RasterBwdArgs& a, cudaStream_t stream) {
  const int64_t blocks = a.B_out * a.num_tiles;
  if (blocks == 0) return;
  const unsigned g = static_cast<unsigned>(blocks);
  launch_bwd<kPixels>(a, g, stream);
}

}  // namespace splax
