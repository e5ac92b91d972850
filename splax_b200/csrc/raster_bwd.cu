// Backward blend: _rasterize_bwd_kernel / _rasterize_bwd_agg_kernel and their depth twins
// (splax/_rasterize/_kernels.py:530-794, 935-1209) with _blend_color_vjp / _blend_depth_vjp
// (:1212-1302).
//
// Recompute-style: one warp per (output image, 16x16 tile); each thread owns eight vertically
// adjacent pixels of one column, advanced as four pairs with packed fp32x2 instructions. The
// walk runs back to front from the tile's largest final_idx over batches of 256 records
// staged in shared memory (plus the flat ids that address the gradients). Each pixel rebuilds
// T by dividing out (1 - alpha), and only entries at or below its own final_idx count. All
// lanes visit the same entry together, so each thread first adds its eight pixels'
// cotangents, then the warp sums the 9 (10 with depth) per-gaussian values with one
// reduce-scatter (~K shuffles instead of 5K) and issues ONE atomic instruction across K
// lanes. Entries to which no pixel of the tile contributes skip the reduction.
//
// The staged conic is pre-scaled (q = -log2(e)/2 * (a, 2b, c)) and log2(opacity) is added to
// the x-term once per record exactly as the forward adds it, so alpha is one ex2 of the same p
// the forward computed; the xy cotangent rescales by -ln 2 to recover the conic.
//
// The 0.999 alpha clamp can only act on a gaussian whose opacity is close to 0.999 (p <=
// log2(opacity) for every entry that takes part). A staged batch without such a record (every
// batch of most scenes) runs a loop that leaves out the clamp and its mask, with identical
// results.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

// the record loop unrolled by two: one record's reduction overlaps the next one's pixel math
// (3.60 -> 3.46 ms; by three 3.51, by four 3.79)
constexpr int kBwdUnroll = 2;

constexpr float kLn2 = 0.693147180559945f;
// Below this opacity alpha = ex2.approx(p) stays under 0.999 for every p <= log2(opacity) (the
// approximation's relative error, about 2^-22, and the rounding of p leave it within 1.001 of
// the opacity).
constexpr float kClampFreeOpacity = 0.998f;

// Two vertically adjacent pixels of one thread, advanced in lock-step with packed fp32x2 math.
struct BwdPair {
  int32_t bf0, bf1;  // bin_final of each pixel
  float2 T, vo0, vo1, vo2, vod;
  // (colour, depth) accumulated behind this gaussian dotted with v_out, plus the
  // background's share t_final * (background . v_out): the term v_alpha subtracts
  float2 behind;
};

// Per-thread sums for the current gaussian, lane-wise over a pixel pair (the two lanes are
// added once per gaussian): colour cotangents, w = ovm * v_alpha and its dy moments, depth.
// v_sigma = -w, so sum v_sigma = -sum w, and the opacity cotangent sum vis * v_alpha is
// sum w / opacity (ov = opacity * vis; both use the same clamp mask).
struct BwdAcc {
  float2 c0, c1, c2, w, wy, wyy, d;
};

// _blend_color_vjp (splax/_rasterize/_kernels.py:1212-1254) for a pixel pair, branch-free:
// a pixel that does not take part (entry past its final_idx, sigma < 0, alpha < 1/255) gets
// alpha 0, leaves T and the colour buffer unchanged and adds exact zeros. The colour buffer
// is kept as its dot product with v_out, plus the background's share: v_alpha = T (c . v_out)
// - ra (buf . v_out + t_final bg . v_out), and buf . v_out grows by (c . v_out) fac.
template <bool DEPTH, bool COUNT, bool CLAMP>
__device__ __forceinline__ bool vjp_pair(BwdPair& s, int32_t idx, float2 p, float2 dy,
                                         float lo, float2 r, float2 g, float2 b, float2 depth,
                                         BwdAcc& acc, unsigned long long& contribs) {
  // p carries log2(opacity) (as in the forward): ov = opacity * 2^(p - lo) = 2^p
  const float2 ov = make_float2(ex2_approx(p.x), ex2_approx(p.y));
  // alpha = min(0.999, ov) < 1/255 exactly when ov < 1/255
  const bool v0 = idx <= s.bf0 && !(p.x > lo) && !(ov.x < kAlphaThreshold);
  const bool v1 = idx <= s.bf1 && !(p.y > lo) && !(ov.y < kAlphaThreshold);
  if constexpr (COUNT) contribs += static_cast<unsigned>(v0) + static_cast<unsigned>(v1);
  // ov of the pixels that take part (0 elsewhere): alpha and the unclamped mask follow from it
  const float2 ovv = make_float2(v0 ? ov.x : 0.0f, v1 ? ov.y : 0.0f);
  const float2 am = CLAMP ? make_float2(fminf(kAlphaMax, ovv.x), fminf(kAlphaMax, ovv.y)) : ovv;
  const float2 om = one_minus2(am);
  const float2 ra = make_float2(__fdividef(1.0f, om.x), __fdividef(1.0f, om.y));
  // a pixel that does not take part has am = 0, om = 1 and ra = rcp.approx(1) = 1 exactly
  // (an exact power of two; checked on B200), so T is left unchanged without a select
  s.T = mul2(s.T, ra);
  const float2 fac = mul2(am, s.T);
  acc.c0 = fma2(s.vo0, fac, acc.c0);
  acc.c1 = fma2(s.vo1, fac, acc.c1);
  acc.c2 = fma2(s.vo2, fac, acc.c2);
  float2 cv = mul2(r, s.vo0);
  cv = fma2(g, s.vo1, cv);
  cv = fma2(b, s.vo2, cv);
  if constexpr (DEPTH) {
    cv = fma2(depth, s.vod, cv);
    acc.d = fma2(s.vod, fac, acc.d);
  }
  const float2 rb = mul2(ra, s.behind);
  const float2 va = fma2(s.T, cv, make_float2(-rb.x, -rb.y));
  s.behind = fma2(cv, fac, s.behind);
  // where the 0.999 clamp is active alpha is constant: no sigma or opacity cotangent
  const float2 ovm = CLAMP ? make_float2(ovv.x <= kAlphaMax ? ovv.x : 0.0f,
                                         ovv.y <= kAlphaMax ? ovv.y : 0.0f)
                          : ovv;
  const float2 w = mul2(ovm, va);
  acc.w = add2(acc.w, w);
  const float2 wy = mul2(w, dy);
  acc.wy = add2(acc.wy, wy);
  acc.wyy = fma2(wy, dy, acc.wyy);
  return v0 || v1;
}

// Eight vertically adjacent pixels per thread (four packed pairs): one warp covers the tile and
// amortises the per-gaussian reduction and record reads over 256 pixels.
constexpr int kPixels = 8;
constexpr int kPairs = kPixels / 2;

template <bool DEPTH, bool COUNT>
__global__ void __launch_bounds__(kBlockSize / kPixels)
raster_bwd_kernel(RasterBwdArgs a) {
  pdl_enter();
  constexpr int kBwdThreads = kBlockSize / kPixels;
  constexpr int K = DEPTH ? 10 : 9;
  unsigned long long evals = 0, contribs = 0;
  unsigned steps = 0, steps_active = 0;  // warp steps (COUNT builds only)
  __shared__ float4 s_r0[kBlockSize];
  __shared__ float4 s_r1[kBlockSize];
  // (b, log2 opacity), or (b, depth, log2 opacity, 0) with depth
  __shared__ std::conditional_t<DEPTH, float4, float2> s_r2[kBlockSize];
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
  const int32_t i0 = tile_y * kBlockWidth + 2 * kPixels * warp + kPixels * (lane >> 4);
  const float px = static_cast<float>(j) + 0.5f;
  const float py0 = static_cast<float>(i0) + 0.5f;

  BwdPair pr[kPairs];
  const float* bg = a.background + 3 * (a.sel_bg ? image_id : 0);
  const float bg0 = bg[0], bg1 = bg[1], bg2 = bg[2];
  int32_t tmax = range_start - 1;
#pragma unroll
  for (int k = 0; k < kPixels; ++k) {
    const int32_t i = i0 + k;
    int32_t bf = range_start - 1;
    float T = 1.0f, vo0 = 0.0f, vo1 = 0.0f, vo2 = 0.0f, vod = 0.0f, tb = 0.0f;
    if (i < a.img_h && j < a.img_w) {
      const int64_t fpix = (geom_image * a.img_h + i) * static_cast<int64_t>(a.img_w) + j;
      bf = min(a.final_idx[fpix], range_end - 1);
      T = a.final_Ts[fpix];
      const int64_t vrow = (image_id * a.img_h + i) % a.vout_rows;
      const float* vo = a.v_out_img + 3 * (vrow * a.img_w + j);
      vo0 = vo[0];
      vo1 = vo[1];
      vo2 = vo[2];
      if constexpr (DEPTH) {
        const int64_t drow = (image_id * a.img_h + i) % a.vdepth_rows;
        vod = a.v_out_depth[drow * a.img_w + j];
      }
      tb = T * (bg0 * vo0 + bg1 * vo1 + bg2 * vo2);
    }
    tmax = max(tmax, bf);
    BwdPair& q = pr[k >> 1];
    if (k & 1) {
      q.bf1 = bf;
      q.T.y = T; q.vo0.y = vo0; q.vo1.y = vo1; q.vo2.y = vo2; q.vod.y = vod; q.behind.y = tb;
    } else {
      q.bf0 = bf;
      q.T.x = T; q.vo0.x = vo0; q.vo1.x = vo1; q.vo2.x = vo2; q.vod.x = vod; q.behind.x = tb;
    }
  }

  // gradient slot this lane owns after a reduce-scatter (fixed by the lane id): output row =
  // staged flat id + my_add, i.e. the (image, gaussian) row, or the gaussian row for the
  // colour / opacity gradients summed over the images
  float* my_base = nullptr;
  int my_stride = 0;
  int64_t my_add = og_base;
  {
    float dummy[K];
#pragma unroll
    for (int k = 0; k < K; ++k) dummy[k] = 0.0f;
    const int c = warp_reduce_scatter<K>(dummy, lane);
    const int64_t to_gaussian = a.sel_geom ? -geom_image * a.n : 0;
    if (c >= 0) {
      if (c < 3) {
        my_base = a.v_colors + c; my_stride = 3;
        if (a.fold_colors) my_add = to_gaussian;
      } else if (c < 6) { my_base = a.v_conic + (c - 3); my_stride = 3; }
      else if (c < 8) { my_base = a.v_xy + (c - 6); my_stride = 2; }
      else if (c == 8) {
        my_base = a.v_opacity; my_stride = 1;
        if (a.fold_opacity) my_add = to_gaussian;
      } else { my_base = a.v_depths; my_stride = 1; }
    }
  }

  // walk starts at the block maximum of final_idx
  const int32_t wmax = __reduce_max_sync(0xffffffffu, tmax);
  if (lane == 0) s_wmax[warp] = wmax;
  __syncthreads();
  int32_t start_idx = s_wmax[0];
#pragma unroll
  for (int w = 1; w < kBwdThreads / 32; ++w) start_idx = max(start_idx, s_wmax[w]);
  const int32_t num_batches = (start_idx - range_start + kBlockSize) / kBlockSize;

  for (int32_t bt = 0; bt < num_batches; ++bt) {
    __syncthreads();  // previous batch's shared reads are complete
    const int32_t batch_end = start_idx - bt * kBlockSize;
    bool high_opacity = false;
#pragma unroll
    for (int h = 0; h < kBlockSize / kBwdThreads; ++h) {
      const int slot = tr + h * kBwdThreads;
      const int32_t src = batch_end - slot;
      if (src >= range_start) {
        const int32_t g = a.gids[src];
        if (g >= 0 && g < a.num_records) {
          const float4* rec = a.records + kRecordFloat4 * static_cast<int64_t>(g);
          s_r0[slot] = rec[0];
          const float4 r1 = rec[1];
          s_r1[slot] = r1;
          high_opacity |= r1.y > kClampFreeOpacity;
          const float4 r2 = rec[2];
          if constexpr (DEPTH) s_r2[slot] = r2;
          else s_r2[slot] = make_float2(r2.x, r2.z);
          s_id[slot] = g;
        } else {  // only after a reported emission error: a transparent record, id 0
          s_r0[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          s_r1[slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if constexpr (DEPTH) s_r2[slot] = make_float4(0.0f, 0.0f, neg_inf(), 0.0f);
          else s_r2[slot] = make_float2(0.0f, neg_inf());
          s_id[slot] = 0;
        }
      }
    }
    // the barrier publishing the batch also tells every lane whether it needs the clamp
    const bool clamp = __syncthreads_or(high_opacity) != 0;
    const int32_t batch_size = min(kBlockSize, batch_end - range_start + 1);
    // entries above every pixel of the tile are skipped as a whole
    const int32_t t_begin = max(0, batch_end - wmax);
    auto walk_batch = [&](auto clamp_tag) {
      constexpr bool kClamp = decltype(clamp_tag)::value;
#pragma unroll kBwdUnroll
    for (int32_t t = t_begin; t < batch_size; ++t) {
      const int32_t idx = batch_end - t;
      const float4 r0 = s_r0[t];
      const auto r2 = s_r2[t];
      float rb, rd, lo;  // b, depth, log2 opacity
      if constexpr (DEPTH) { rb = r2.x; rd = r2.y; lo = r2.z; }
      else { rb = r2.x; rd = 0.0f; lo = r2.y; }
      if constexpr (COUNT) {
#pragma unroll
        for (int q = 0; q < kPairs; ++q)
          evals += static_cast<unsigned>(idx <= pr[q].bf0) + static_cast<unsigned>(idx <= pr[q].bf1);
        ++steps;
      }
      const float4 r1 = s_r1[t];  // qc, opacity, r, g
      const float dx = r0.x - px;
      const float dy0 = r0.y - py0;
      // the x-term carries log2(opacity): one explicit FMA, as the forward computes it
      const float2 qxx = splat2(fmaf(r0.z * dx, dx, lo)), qbx = splat2(r0.w * dx),
                   qc = splat2(r1.x);
      const float2 cr = splat2(r1.z), cg = splat2(r1.w), cb = splat2(rb), cd = splat2(rd);
      BwdAcc acc;
      acc.c0 = acc.c1 = acc.c2 = acc.w = acc.wy = acc.wyy = acc.d = make_float2(0.0f, 0.0f);
      bool any = false;
#pragma unroll
      for (int q = 0; q < kPairs; ++q) {
        const float2 dy = add2(splat2(dy0), make_float2(-2.0f * q, -2.0f * q - 1.0f));
        const float2 p = fma2(fma2(qc, dy, qbx), dy, qxx);
        any |= vjp_pair<DEPTH, COUNT, kClamp>(pr[q], idx, p, dy, lo, cr, cg, cb, cd, acc,
                                              contribs);
      }
      if (__ballot_sync(0xffffffffu, any) == 0u) continue;
      if constexpr (COUNT) ++steps_active;
      // per-thread cotangents from the sums (v_sigma = -w): the conic and xy terms use the
      // second moments; (a, b, c) = -ln2 (2 qa, qb, 2 qc) recovers the unscaled conic
      const float W = acc.w.x + acc.w.y, WY = acc.wy.x + acc.wy.y, WYY = acc.wyy.x + acc.wyy.y;
      const float sxn = W * dx;  // -sum v_sigma dx
      const float a2n = 2.0f * kLn2 * r0.z, bqn = kLn2 * r0.w, c2n = 2.0f * kLn2 * r1.x;
      float v[K];
      v[0] = acc.c0.x + acc.c0.y;
      v[1] = acc.c1.x + acc.c1.y;
      v[2] = acc.c2.x + acc.c2.y;
      v[3] = -0.5f * sxn * dx;
      v[4] = -WY * dx;
      v[5] = -0.5f * WYY;
      v[6] = fmaf(a2n, sxn, bqn * WY);
      v[7] = fmaf(bqn, sxn, c2n * WY);
      v[8] = __fdividef(W, r1.y);  // opacity > 0 whenever a lane of the warp contributes
      if constexpr (DEPTH) v[9] = acc.d.x + acc.d.y;
      warp_reduce_scatter<K>(v, lane);
      if (my_base != nullptr && v[0] != 0.0f) {
        atomicAdd(my_base + (s_id[t] + my_add) * my_stride, v[0]);
      }
    }
    };
    if (clamp) walk_batch(std::true_type{});
    else walk_batch(std::false_type{});
  }
  if constexpr (COUNT) {
    evals = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(evals));
    contribs = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(contribs));
    if (lane == 0) {
      atomicAdd(&a.work[0], evals);
      atomicAdd(&a.work[1], contribs);
      atomicAdd(&a.work[2], static_cast<unsigned long long>(steps));
      atomicAdd(&a.work[3], static_cast<unsigned long long>(steps_active));
    }
  }
}

void launch_bwd(const RasterBwdArgs& a, unsigned g, cudaStream_t stream) {
  constexpr int nt = kBlockSize / kPixels;
  if (a.v_out_depth) {
    if (a.work) launch_pdl(raster_bwd_kernel<true, true>, g, nt, 0, stream, a);
    else launch_pdl(raster_bwd_kernel<true, false>, g, nt, 0, stream, a);
  } else {
    if (a.work) launch_pdl(raster_bwd_kernel<false, true>, g, nt, 0, stream, a);
    else launch_pdl(raster_bwd_kernel<false, false>, g, nt, 0, stream, a);
  }
}

}  // namespace

void launch_raster_bwd(const RasterBwdArgs& a, cudaStream_t stream) {
  const int64_t blocks = a.B_out * a.num_tiles;
  if (blocks == 0) return;
  const unsigned g = static_cast<unsigned>(blocks);
  launch_bwd(a, g, stream);
}

}  // namespace splax
