// Intersection keys, their radix sort and the per-tile bin edges: the device half of
// sort_and_bin (splax/_rasterize/_sort/_sort.py:29-171).
//
//  depth min/max   per-image [dmin, dmax] of visible depths (_sort/_kernels.py:31-73), a
//                  warp-reduced atomic min/max on order-preserving integers.
//  pair order     the B*n pairs sorted stably by (image, depth key), and the exclusive scan
//                  of their tile counts in that order.
//  emission        the ellipse tile walk once more per visible pair, in sorted pair order
//                  (_kernels.py:76-211), writing (image | tile) bin keys and flat ids, and
//                  packing the pair's blend record (xy, conic, opacity, colour, depth).
//  radix sort      stable LSD onesweep (used for both sorts): one upfront histogram pass, then one
//                  kernel per 8-bit digit that ranks keys with warp match groups, resolves the
//                  tile's global digit offsets by a decoupled look-back (bounded spin) and
//                  scatters through shared memory so the global writes coalesce per digit.
//                  Only the significant key bits are sorted.
//  bin edges       [start, end) per (image, tile) from the sorted keys (_kernels.py:214-269).
//
// Compiled with --fmad=false so the emitted walk and quantised depths match the projection's
// count and the C oracle bit for bit.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

// ------------------------------------------------------------------ zero fill
struct ClearArgs {
  uint32_t* p[kClearMaxSpans];
  int64_t words[kClearMaxSpans];
  int count;
};
constexpr int kClearThreads = 256;
constexpr size_t kSelfClearBytes = 8u << 20;

__global__ void __launch_bounds__(kClearThreads) clear_kernel(ClearArgs a) {
  pdl_enter();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kClearThreads;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kClearThreads + threadIdx.x;
  for (int r = 0; r < a.count; ++r) {
    uint32_t* p = a.p[r];
    const int64_t w = a.words[r];
    // words up to the first 16-byte boundary, the 16-byte body, the remaining words
    const int64_t lead = (16 - static_cast<int64_t>(reinterpret_cast<uintptr_t>(p) & 15)) & 15;
    const int64_t head = lead / 4 < w ? lead / 4 : w;
    if (t0 < head) p[t0] = 0u;
    uint4* body = reinterpret_cast<uint4*>(p + head);
    const int64_t n4 = (w - head) / 4;
    for (int64_t i = t0; i < n4; i += stride) body[i] = make_uint4(0u, 0u, 0u, 0u);
    const int64_t tail0 = head + 4 * n4;
    if (t0 < w - tail0) p[tail0 + t0] = 0u;
  }
}

// ------------------------------------------------------------------ depth min / max
constexpr int kMmThreads = 256;
constexpr int kMmItems = 16;

__global__ void seed_minmax_kernel(int32_t* mm, int32_t B) {
  pdl_enter();
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    mm[2 * b] = float_to_ordered(1.0e30f);
    mm[2 * b + 1] = float_to_ordered(-1.0e30f);
  }
}

// Per-image [min, max] of the visible pairs' depths (as ordered ints). Each thread takes 16
// consecutive pairs with all its loads issued up front (four 16-byte loads of radii and of
// depths when the run is whole and aligned), so the kernel streams at memory speed instead of
// waiting on one dependent load per pair. With n >= 16 a thread's run spans at most two images.
__device__ __forceinline__ void mm_flush(int32_t* mm, int64_t im, int32_t lo, int32_t hi) {
  if (lo <= hi) {
    atomicMin(&mm[2 * im], lo);
    atomicMax(&mm[2 * im + 1], hi);
  }
}

__global__ void __launch_bounds__(kMmThreads)
depth_minmax_kernel(const float* __restrict__ depths, const int32_t* __restrict__ radii,
                    int64_t total, int64_t n, int32_t* mm) {
  pdl_enter();
  const int64_t base = (static_cast<int64_t>(blockIdx.x) * kMmThreads + threadIdx.x) * kMmItems;
  int32_t r[kMmItems];
  float d[kMmItems];
  if (base + kMmItems <= total) {
    const int4* r4 = reinterpret_cast<const int4*>(radii + base);
    const float4* d4 = reinterpret_cast<const float4*>(depths + base);
#pragma unroll
    for (int v = 0; v < kMmItems / 4; ++v) {
      const int4 a = __ldg(r4 + v);
      const float4 b = __ldg(d4 + v);
      r[4 * v] = a.x; r[4 * v + 1] = a.y; r[4 * v + 2] = a.z; r[4 * v + 3] = a.w;
      d[4 * v] = b.x; d[4 * v + 1] = b.y; d[4 * v + 2] = b.z; d[4 * v + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < kMmItems; ++k) {
      const bool in = base + k < total;
      r[k] = in ? radii[base + k] : 0;
      d[k] = in ? depths[base + k] : 0.0f;
    }
  }
  // the run's first image and where the next one starts (n >= kMmItems: at most one boundary)
  const int64_t im0 = base < total ? base / n : -1;
  const int64_t cut = (im0 + 1) * n - base;  // items before the boundary
  int32_t lo0 = 0x7fffffff, hi0 = static_cast<int32_t>(0x80000000u);
  int32_t lo1 = 0x7fffffff, hi1 = static_cast<int32_t>(0x80000000u);
#pragma unroll
  for (int k = 0; k < kMmItems; ++k) {
    if (r[k] <= 0) continue;
    const int32_t o = float_to_ordered(d[k]);
    if (k < cut) {
      lo0 = min(lo0, o);
      hi0 = max(hi0, o);
    } else {
      lo1 = min(lo1, o);
      hi1 = max(hi1, o);
    }
  }
  // one atomic pair per warp when every lane's run lies in one image, per lane otherwise
  const long long first = __shfl_sync(0xffffffffu, static_cast<long long>(im0), 0);
  const bool one_image = __all_sync(0xffffffffu, im0 == first && (im0 < 0 || cut >= kMmItems));
  if (one_image) {
    const int32_t wlo = __reduce_min_sync(0xffffffffu, lo0);
    const int32_t whi = __reduce_max_sync(0xffffffffu, hi0);
    if ((threadIdx.x & 31) == 0 && first >= 0) mm_flush(mm, first, wlo, whi);
  } else if (im0 >= 0) {
    mm_flush(mm, im0, lo0, hi0);
    if (cut < kMmItems) mm_flush(mm, im0 + 1, lo1, hi1);
  }
}

// Any n (also n < 16): one dependent pass per pair; used only when a run could span more
// than two images.
__global__ void __launch_bounds__(kMmThreads)
depth_minmax_small_n_kernel(const float* __restrict__ depths, const int32_t* __restrict__ radii,
                            int64_t total, int64_t n, int32_t* mm) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * kMmThreads + threadIdx.x;
  if (idx >= total || radii[idx] <= 0) return;
  const int32_t o = float_to_ordered(depths[idx]);
  mm_flush(mm, idx / n, o, o);
}

// ------------------------------------------------------------------ depth-first ordering
// The reference sorts every intersection by the key (image | tile | depth) (_sort/_kernels.py
// :76-211), stably over emission order (ascending flat id). Within one (image, tile) bin that
// order is (depth key, flat id). The same order arises from two stable sorts: the B*n pairs by
// (image, depth key), then -- after emitting each pair's tiles in that order -- the
// intersections by their (image | tile) field alone. The first sort touches B*n pairs, the
// second only the image and tile bits, instead of every depth bit of every intersection.

// Largest per-image span of visible depth bit patterns (64-bit key mode): the pair key stores
// depth bits relative to the image's minimum, which orders positive floats like their values.
__global__ void depth_span_kernel(const int32_t* mm, int32_t B, unsigned* span_out) {
  pdl_enter();
  unsigned span = 0;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int32_t lo = mm[2 * b], hi = mm[2 * b + 1];
    if (lo <= hi) span = max(span, static_cast<unsigned>(hi - lo));
  }
  span = __reduce_max_sync(0xffffffffu, span);
  __shared__ unsigned s_span[32];
  if ((threadIdx.x & 31) == 0) s_span[threadIdx.x >> 5] = span;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned m = 0;
    for (int w = 0; w < (blockDim.x + 31) / 32; ++w) m = max(m, s_span[w]);
    *span_out = m;
  }
}

// Per pair, in flat order (coalesced): the pair key (image | depth key), its tile count, its
// 32-byte walk record for the emission and (when blending) its 48-byte blend record. A pair
// that hits no tile gets the all-ones key, which no real key reaches (pair keys widen to 64
// bits from 32 significant bits up): the depth sort's histogram and first pass skip it, so only
// the V pairs that hit a tile are sorted, and V stays in device memory.
//  packed keys: the reference's quantised depth (_sort/_kernels.py:116-124)
//  wide keys:   float bits - the image's minimum visible float bits (orders like the value)
constexpr int kPrepThreads = 256;

template <typename K>
__device__ __forceinline__ bool prep_one(const PairKeyArgs& a, int64_t idx, K& key) {
  const int64_t bid = idx / a.n;
  const bool live = a.radii[idx] > 0;
  uint64_t dk = 0;
  const float depth = a.depths[idx];
  if (live) {
    if (a.packed) {
      const float dmin = ordered_to_float(a.depth_mm[2 * bid]);
      const float drange = ordered_to_float(a.depth_mm[2 * bid + 1]) - dmin;
      const int32_t qmax = static_cast<int32_t>((1u << a.depth_bits) - 1u);
      const float maxq = static_cast<float>(qmax);
      if (drange > 0.0f) {
        const float f = (depth - dmin) / drange;
        dk = static_cast<uint64_t>(imin(imax(f2i(f * maxq), 0), qmax));
      }
    } else {
      const int32_t dbits = __float_as_int(depth);
      // the reference sign-extends a negative depth into the image and tile fields
      if (dbits < 0) atomicOr(a.err, kErrNegativeDepthKey);
      dk = static_cast<uint32_t>(dbits - a.depth_mm[2 * bid]);
    }
  }
  key = static_cast<K>((static_cast<uint64_t>(bid) << a.key_shift) | dk);
  const int64_t hi = static_cast<uint32_t>(a.cum[idx]);
  const int64_t lo = idx > 0 ? static_cast<int64_t>(static_cast<uint32_t>(a.cum[idx - 1])) : 0;
  int64_t count = hi - lo;
  if (!live) {
    // the reference emits nothing for a culled pair; its cum range must then be empty
    if (count != 0) atomicOr(a.err, kErrEmitCount);
    count = 0;
  }
  a.counts[idx] = static_cast<int32_t>(count);
  if (!live) return false;
  const float x = a.xys[2 * idx], y = a.xys[2 * idx + 1];
  const float ca = a.conics[3 * idx], cb = a.conics[3 * idx + 1], cc = a.conics[3 * idx + 2];
  const float mop = a.map_opacities[idx % a.map_opac_rows];
  float4* w = a.walk + 2 * idx;
  w[0] = make_float4(x, y, ca, cb);
  w[1] = make_float4(cc, iso_level(mop), __int_as_float(static_cast<int32_t>(bid)),
                     __int_as_float(static_cast<int32_t>(count)));
  if (a.records) {
    const int64_t ci = idx % a.color_rows;
    const float op = a.opacities[idx % a.opac_rows];
    float4* rec = a.records + kRecordFloat4 * idx;
    // conic pre-scaled for the blends' base-2 exponent: q = -log2(e)/2 * (a, 2b, c)
    rec[0] = make_float4(x, y, -kHalfLog2e * ca, -kLog2e * cb);
    rec[1] = make_float4(-kHalfLog2e * cc, op, a.colors[3 * ci], a.colors[3 * ci + 1]);
    // log2 of the blend opacity, added to the blends' exponent (alpha = 2^p); a zero or
    // negative opacity is never blended (alpha < 1/255), so it gets -inf: alpha 0
    rec[2] = make_float4(a.colors[3 * ci + 2], depth, op > 0.0f ? log2f(op) : neg_inf(), 0.0f);
  }
  return count > 0;
}

template <typename K>
__global__ void __launch_bounds__(kPrepThreads) pair_prep_kernel(PairKeyArgs a, K* keys,
                                                                 int32_t* vals) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * kPrepThreads + threadIdx.x;
  if (idx >= a.total) return;
  K kk = K(0);
  const bool vis = prep_one<K>(a, idx, kk);
  keys[idx] = vis ? kk : static_cast<K>(~K(0));  // all ones: left out of the depth sort
  vals[idx] = static_cast<int32_t>(idx);
}

// Exclusive scan of the tile counts in sorted pair order, one pass with a decoupled look-back
// (bounded spin).
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;  // the 16-byte loads and stores below assume 8

__global__ void __launch_bounds__(kScanThreads)
sorted_offsets_kernel(const int32_t* __restrict__ perm, const int32_t* __restrict__ counts,
                      int64_t total, const int32_t* dtotal, int32_t* __restrict__ offsets,
                      unsigned long long* status, int* ticket, unsigned* err) {
  pdl_enter();
  __shared__ int s_tile;
  __shared__ long long s_warp[kScanThreads / 32];
  __shared__ long long s_prefix;
  if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1);
  __syncthreads();
  const int64_t tile = s_tile;
  if (dtotal) total = *dtotal;  // grid sized for the largest count; surplus tiles leave
  if (tile * kScanThreads * kScanItems >= total) return;
  const int64_t base = tile * kScanThreads * kScanItems + static_cast<int64_t>(threadIdx.x) * kScanItems;
  long long c[kScanItems];
  long long tsum = 0;
  const bool full = base + kScanItems <= total;  // whole run: two 16-byte loads of perm
  int32_t pm[kScanItems];
  if (full) {
    const int4 p0 = *reinterpret_cast<const int4*>(perm + base);
    const int4 p1 = *reinterpret_cast<const int4*>(perm + base + 4);
    pm[0] = p0.x; pm[1] = p0.y; pm[2] = p0.z; pm[3] = p0.w;
    pm[4] = p1.x; pm[5] = p1.y; pm[6] = p1.z; pm[7] = p1.w;
  } else {
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) pm[k] = base + k < total ? perm[base + k] : -1;
  }
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const long long v = pm[k] >= 0 ? counts[pm[k]] : 0;
    c[k] = v;
    tsum += v;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long inc = tsum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long o = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += o;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  long long wpre = 0;
  for (int w = 0; w < warp; ++w) wpre += s_warp[w];
  if (warp == 0) {
    long long agg = 0;
    for (int w = 0; w < kScanThreads / 32; ++w) agg += s_warp[w];
    long long prefix = 0;
    if (tile == 0) {
      if (lane == 0) st_relaxed(&status[0], kLookbackInc | static_cast<unsigned long long>(agg));
    } else {
      if (lane == 0) st_relaxed(&status[tile], kLookbackAgg | static_cast<unsigned long long>(agg));
      prefix = warp_lookback(status, tile, err);
      if (lane == 0)
        st_relaxed(&status[tile], kLookbackInc | static_cast<unsigned long long>(prefix + agg));
    }
    if (lane == 0) s_prefix = prefix;
  }
  __syncthreads();
  long long run = s_prefix + wpre + inc - tsum;
  int32_t o[kScanItems];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    o[k] = static_cast<int32_t>(run);
    run += c[k];
  }
  if (full) {
    *reinterpret_cast<int4*>(offsets + base) = make_int4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<int4*>(offsets + base + 4) = make_int4(o[4], o[5], o[6], o[7]);
  } else {
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
      if (base + k < total) offsets[base + k] = o[k];
  }
}

// Emission in sorted pair order, warp-cooperative: each warp takes 32 consecutive sorted pairs
// and produces their (image | tile) bin keys and flat ids at the pairs' offsets.
//  1. Each lane sets up its pair's ellipse walk (the count projection made) and shares it
//     (warp_walk_share).
//  2. Rows are taken 32 at a time, one per lane (warp_walk_row: bit-identical to the
//     sequential walk).
//  3. The rows' tile runs are expanded 32 tiles at a time: each lane finds its row by binary
//     lifting over the width scan, so consecutive lanes write consecutive keys.
// The pairs' offsets must chain (each pair starts where the previous one ends, as the scan of
// the counts gives); a mismatch with the walk sets kErrEmitCount, and no write leaves
// [0, count).
constexpr int kEmitWarps = 4;
constexpr int kEmitThreads = 32 * kEmitWarps;

__global__ void __launch_bounds__(kEmitThreads) emit_sorted_kernel(EmitArgs a) {
  pdl_enter();
  __shared__ WarpWalk s_walk[kEmitWarps];
  __shared__ int32_t s_x[kEmitWarps][3][32];  // flat id, offset, image bits of each lane's pair
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const int64_t V = a.dtotal ? static_cast<int64_t>(*a.dtotal) : a.total;
  const int64_t first = (static_cast<int64_t>(blockIdx.x) * kEmitWarps + wi) * 32;
  if (first >= V) return;  // warp-uniform
  const int64_t i = first + lane;
  // ---- 1. per-pair setup
  int32_t cnt = 0, off = 0, idx = -1;
  Ellipse e{};
  int32_t bid = 0;
  if (i < V) {
    idx = a.perm[i];
    off = a.offsets[i];
    if (idx >= 0 && idx < a.total) cnt = a.counts[idx];
    if (cnt > 0) {
      const float4 w0 = a.walk[2 * static_cast<int64_t>(idx)];
      const float4 w1 = a.walk[2 * static_cast<int64_t>(idx) + 1];
      bid = __float_as_int(w1.z);
      ellipse_init(w0.z, w0.w, w1.x, w1.y, w0.x, w0.y, a.tbx, a.tby, e);
    }
  }
  s_x[wi][0][lane] = idx;
  s_x[wi][1][lane] = off;
  s_x[wi][2][lane] = static_cast<int32_t>(static_cast<uint32_t>(bid) << a.tile_n_bits);
  int rexc;
  const int rows = warp_walk_share(s_walk[wi], lane, e, rexc);
  const int last = V - first > 32 ? 31 : static_cast<int>(V - 1 - first);
  const int64_t out0 = __shfl_sync(0xffffffffu, off, 0);
  const int64_t out_end = __shfl_sync(0xffffffffu, off + cnt, last);
  bool bad = false;
  int64_t done = 0;  // tiles written by the earlier row chunks
  const WarpWalk& W = s_walk[wi];
  // ---- 2. rows, 32 at a time
  for (int c0 = 0; c0 < rows; c0 += 32) {
    const int r = c0 + lane;
    int ow, u;
    int32_t mn, mx;
    warp_walk_row(W, lane, rexc, r, rows, ow, u, mn, mx);
    const bool has = r < rows;
    const int w = has ? max(mx - mn, 0) : 0;
    int winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += v;
    }
    const int wexc = winc - w;
    const int total = __shfl_sync(0xffffffffu, winc, 31);
    const int64_t pos = out0 + done + wexc;
    if (has && u == W.n[0][ow] && pos != s_x[wi][1][ow]) bad = true;  // offsets must chain
    const bool isY = W.n[3][ow] != 0;
    const uint32_t key0 = static_cast<uint32_t>(s_x[wi][2][ow]) |
                          static_cast<uint32_t>(isY ? u * a.tbx + mn : mn * a.tbx + u);
    const int kstep = isY ? 1 : a.tbx;
    const int32_t val = s_x[wi][0][ow];
    // ---- 3. expand the chunk's tiles, 32 at a time
    for (int q0 = 0; q0 < total; q0 += 32) {
      const int q = q0 + lane;
      const int rr = lift_find(wexc, q);
      const int k = q - __shfl_sync(0xffffffffu, wexc, rr);
      const uint32_t kk = __shfl_sync(0xffffffffu, key0, rr);
      const int ks = __shfl_sync(0xffffffffu, kstep, rr);
      const int32_t vv = __shfl_sync(0xffffffffu, val, rr);
      const long long p0 = __shfl_sync(0xffffffffu, static_cast<long long>(pos), rr);
      if (q < total) {
        const int64_t p = p0 + k;
        if (p >= 0 && p < a.count) {
          a.keys[p] = kk + static_cast<uint32_t>(k * ks);
          a.vals[p] = vv;
        } else {
          bad = true;
        }
      }
    }
    done += total;
  }
  if (out0 + done != out_end) bad = true;
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(a.err, kErrEmitCount);
}

// The reference's own sort keys for the sorted order (for the parity entry point only):
// packed (bin << depth_bits) | quantised depth, wide (bin << 32) | depth bits.
__global__ void reference_keys_kernel(const uint32_t* __restrict__ bin_keys,
                                      const int32_t* __restrict__ gids, int64_t count,
                                      PairKeyArgs a, int64_t* out) {
  pdl_enter();
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= count) return;
  const int64_t idx = gids[p];
  const int64_t bid = idx / a.n;
  const float depth = a.depths[idx];
  uint64_t key;
  if (a.packed) {
    uint32_t q = 0;
    const float dmin = ordered_to_float(a.depth_mm[2 * bid]);
    const float drange = ordered_to_float(a.depth_mm[2 * bid + 1]) - dmin;
    const int32_t qmax = static_cast<int32_t>((1u << a.depth_bits) - 1u);
    if (drange > 0.0f) {
      const float f = (depth - dmin) / drange;
      q = static_cast<uint32_t>(imin(imax(f2i(f * static_cast<float>(qmax)), 0), qmax));
    }
    key = (static_cast<uint64_t>(bin_keys[p]) << a.depth_bits) | q;
  } else {
    key = (static_cast<uint64_t>(bin_keys[p]) << 32) |
          static_cast<uint64_t>(static_cast<int64_t>(__float_as_int(depth)));
  }
  out[p] = static_cast<int64_t>(key);
}

// ------------------------------------------------------------------ onesweep radix sort
constexpr int kSortThreads = 512;
constexpr int kItems32 = 12;  // 6144 keys per tile for 32-bit keys
constexpr int kItems64 = 8;   // 4096 keys per tile for 64-bit keys
constexpr int kHistThreads = 256;
constexpr int kHistItems = 32;
constexpr int kRadixHistWords = 2048;  // per histogram array: passes x digits

// Upfront digit histograms of every pass in one read of the keys (RB-bit digits: up to 8 passes
// of 8 bits or 4 of 9): four sets of shared counters, each shared by two warps (less
// same-address contention than one block-wide set), 16-byte loads, then one global atomic per
// (pass, digit) and block.
template <typename K, int RB>
__global__ void __launch_bounds__(kHistThreads)
radix_hist_kernel(const K* __restrict__ keys, int64_t count, bool filter, int passes,
                  uint32_t* hist) {
  pdl_enter();
  constexpr int kSets = 4;
  constexpr int D = 1 << RB;
  constexpr int kMaxPasses = kRadixHistWords / D;
  constexpr int kVec = 16 / sizeof(K);  // keys per 16-byte load
  __shared__ uint32_t s[kSets][kMaxPasses][D];
  const int warp = (threadIdx.x >> 5) & (kSets - 1);
  for (int i = threadIdx.x; i < kSets * kMaxPasses * D; i += kHistThreads) (&s[0][0][0])[i] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kHistThreads * kHistItems;
  const int64_t end = min(count, base + static_cast<int64_t>(kHistThreads) * kHistItems);
  auto add = [&](uint64_t key) {
    if (filter && key == static_cast<uint64_t>(static_cast<K>(~K(0)))) return;  // left out
    for (int p = 0; p < passes; ++p) atomicAdd(&s[warp][p][(key >> (RB * p)) & (D - 1)], 1u);
  };
  if (end - base == static_cast<int64_t>(kHistThreads) * kHistItems) {
    const uint4* v = reinterpret_cast<const uint4*>(keys + base);
#pragma unroll 2
    for (int j = 0; j < kHistItems / kVec; ++j) {
      const uint4 q = v[j * kHistThreads + threadIdx.x];
      if constexpr (sizeof(K) == 4) {
        add(q.x); add(q.y); add(q.z); add(q.w);
      } else {
        add((static_cast<uint64_t>(q.y) << 32) | q.x);
        add((static_cast<uint64_t>(q.w) << 32) | q.z);
      }
    }
  } else {
    for (int64_t i = base + threadIdx.x; i < end; i += kHistThreads)
      add(static_cast<uint64_t>(keys[i]));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * D; i += kHistThreads) {
    const int p = i >> RB, d = i & (D - 1);
    uint32_t c = 0;
#pragma unroll
    for (int w = 0; w < kSets; ++w) c += s[w][p][d];
    if (c) atomicAdd(&hist[p * D + d], c);
  }
}

// Exclusive scan over the block (NT threads); s_warp holds NT/32 words.
template <int NT>
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t o = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += o;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  uint32_t wpre = 0;
  for (int w = 0; w < warp; ++w) wpre += s_warp[w];
  return wpre + inc - v;
}

// exclusive scan of each pass's D-digit histogram (D threads): offsets[p][d]; with total_out,
// pass 0 also writes the number of keys sorted
template <int D>
__global__ void __launch_bounds__(D)
radix_scan_kernel(const uint32_t* hist, uint32_t* offsets, int32_t* total_out) {
  pdl_enter();
  __shared__ uint32_t s_warp[D / 32];
  const int p = blockIdx.x;
  const uint32_t v = hist[p * D + threadIdx.x];
  const uint32_t ex = block_exclusive_scan<D>(v, s_warp);
  offsets[p * D + threadIdx.x] = ex;
  if (total_out && p == 0 && threadIdx.x == D - 1) *total_out = static_cast<int32_t>(ex + v);
}

// FILTER (first pass of the depth sort): all-ones keys are neither ranked nor written, so the
// output holds only the other keys, in stable order. RB: digit bits (8 or 9; NT >= 2^RB).
template <typename K, int ITEMS, int NT, bool FILTER, int RB>
__global__ void __launch_bounds__(NT)
onesweep_kernel(const K* __restrict__ kin, const int32_t* __restrict__ vin, K* __restrict__ kout,
                int32_t* __restrict__ vout, int64_t count, const int32_t* dcount, int shift,
                const uint32_t* __restrict__ goff, unsigned long long* status, int* tile_counter,
                unsigned* err, unsigned long long* clear_next) {
  pdl_enter();
  constexpr int TILE = NT * ITEMS;
  constexpr int kSortWarps = NT / 32;
  constexpr int D = 1 << RB;
  static_assert(NT >= D, "one thread per digit");
  __shared__ uint32_t s_wh[kSortWarps][D];
  // a digit's lanes are found through a shared word per (warp, digit): atomicOr of the lane bits,
  // a quarter of the instructions of one ballot per digit bit (sort 1.07 -> 0.97 ms per step).
  // The words live in the dynamic buffer, which the ranking does not otherwise use (the staged
  // keys and values are written after it).
  static_assert(kSortWarps * D * sizeof(uint32_t) <= TILE * (sizeof(K) + sizeof(int32_t)),
                "the digit words fit in the staging buffer");
  __shared__ uint32_t s_bx[D];
  __shared__ long long s_gb[D];
  __shared__ uint32_t s_warp[kSortWarps];
  __shared__ int s_tile;
  __shared__ int s_tile_keys;
  extern __shared__ __align__(16) unsigned char s_raw[];
  uint32_t* s_match = reinterpret_cast<uint32_t*>(s_raw);  // [kSortWarps][D], ranking only
  K* s_keys = reinterpret_cast<K*>(s_raw);
  int32_t* s_vals = reinterpret_cast<int32_t*>(s_raw + TILE * sizeof(K));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kSortWarps * D; i += NT) (&s_wh[0][0])[i] = 0;
  for (int i = tid; i < kSortWarps * D; i += NT) s_match[i] = 0;
  if (tid == 0) s_tile = atomicAdd(tile_counter, 1);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t base = tile * TILE;
  // the previous pass has completed (pdl_enter): clear its look-back words, which the next pass
  // reuses, this tile's row of them (every tile of the grid, surplus ones included)
  if (clear_next != nullptr && tid < D) clear_next[tile * D + tid] = 0ull;
  if (dcount) count = *dcount;  // grid sized for the largest count; surplus tiles leave
  if (base >= count) return;
  const int64_t rem = count - base;
  const int nvalid = rem < TILE ? static_cast<int>(rem) : TILE;
  const int warp_base = warp * 32 * ITEMS;
  const unsigned lt_mask = (1u << lane) - 1u;

  K k[ITEMS];
  int32_t val[ITEMS];
  uint32_t rank[ITEMS];
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int pos = warp_base + it * 32 + lane;
    const bool valid = pos < nvalid;
    k[it] = valid ? kin[base + pos] : K(0);
    val[it] = valid ? vin[base + pos] : 0;
  }
  // stable warp-level ranking: keys of one digit keep their input order (iteration, lane).
  // The lowest lane of each digit group adds the group's size to the warp's counter with one
  // shared atomic and broadcasts the old value; the atomics of successive iterations are
  // independent instructions executed in order, so the iterations pipeline.
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int pos = warp_base + it * 32 + lane;
    const bool valid = pos < nvalid && (!FILTER || k[it] != static_cast<K>(~K(0)));
    const uint32_t d = static_cast<uint32_t>(static_cast<uint64_t>(k[it]) >> shift) & (D - 1);
    // lanes holding the same digit: intersect one ballot per digit bit (cheaper than a
    // match instruction over up to 32 distinct digits); invalid lanes match nobody
    // lanes holding the same digit: each ORs its bit into the digit's word, reads the word
    // back, and the group's lowest lane clears it for the next item
    uint32_t* word = s_match + warp * D + d;
    if (valid) atomicOr(word, 1u << lane);
    __syncwarp();
    const unsigned peers = valid ? *word : (1u << lane);
    __syncwarp();
    if (valid && (peers & lt_mask) == 0) *word = 0;
    __syncwarp();
    const int leader = __ffs(peers) - 1;
    uint32_t prev = 0;
    if (valid && lane == leader) prev = atomicAdd(&s_wh[warp][d], __popc(peers));
    prev = __shfl_sync(0xffffffffu, prev, leader);
    rank[it] = prev + __popc(peers & lt_mask);
  }
  __syncthreads();
  // per digit (threads 0..255): warp exclusive offsets, the block's count, the look-back
  uint32_t sum = 0;
  long long prefix = 0;
  if (tid < D) {
    const int dg = tid;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t c = s_wh[w][dg];
      s_wh[w][dg] = sum;
      sum += c;
    }
    unsigned long long* st = status + tile * D + dg;
    if (tile == 0) {
      st_relaxed(st, kLookbackInc | sum);
    } else {
      st_relaxed(st, kLookbackAgg | sum);
      // walk back kLookAhead predecessors per round trip: sum aggregates up to the nearest
      // inclusive prefix; a predecessor that has published nothing yet is re-read (bounded)
      constexpr int kLookAhead = 4;
      int64_t j = tile - 1;
      long long spins = 0;
      bool done = false;
      while (!done && j >= 0) {
        unsigned long long w[kLookAhead];
#pragma unroll
        for (int q = 0; q < kLookAhead; ++q)
          w[q] = j - q >= 0 ? ld_relaxed(status + (j - q) * D + dg) : kLookbackInc;
        int used = 0;
#pragma unroll
        for (int q = 0; q < kLookAhead; ++q) {
          if (done || used < q) continue;  // stopped at an unpublished word
          const unsigned long long flag = w[q] & ~kLookbackMask;
          if (flag == 0) continue;
          prefix += static_cast<long long>(w[q] & kLookbackMask);
          used = q + 1;
          if (flag == kLookbackInc) done = true;
        }
        j -= used;
        if (!done && used < kLookAhead) {  // waiting on tile j
          if (++spins > kSpinLimit) {
            atomicOr(err, kErrLookbackTimeout);
            break;
          }
        }
      }
      st_relaxed(st, kLookbackInc | (static_cast<unsigned long long>(prefix) + sum));
    }
  }
  const uint32_t excl = block_exclusive_scan<NT>(sum, s_warp);
  if (tid == D - 1) s_tile_keys = static_cast<int>(excl + sum);  // keys this tile writes
  if (tid < D) {
    s_bx[tid] = excl;
    s_gb[tid] = static_cast<long long>(goff[tid]) + prefix - static_cast<long long>(excl);
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int pos = warp_base + it * 32 + lane;
    if (pos < nvalid && (!FILTER || k[it] != static_cast<K>(~K(0)))) {
      const uint32_t d = static_cast<uint32_t>(static_cast<uint64_t>(k[it]) >> shift) & (D - 1);
      const uint32_t lpos = s_bx[d] + s_wh[warp][d] + rank[it];
      s_keys[lpos] = k[it];
      s_vals[lpos] = val[it];
    }
  }
  __syncthreads();
  const int tile_keys = s_tile_keys;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    const int p = j * NT + tid;
    if (p < tile_keys) {
      const K kk = s_keys[p];
      const uint32_t d = static_cast<uint32_t>(static_cast<uint64_t>(kk) >> shift) & (D - 1);
      const long long dst = s_gb[d] + p;
      if (dst >= 0 && dst < count) {
        kout[dst] = kk;
        vout[dst] = s_vals[p];
      } else {
        atomicOr(err, kErrLookbackTimeout);
      }
    }
  }
}

// ------------------------------------------------------------------ bin edges
// Eight sorted keys per thread (two 16-byte loads); the key before the first comes from the
// previous lane by shuffle (global load for lane 0). The edge logic per index is the
// reference's, including its index-0 early return before the last-index test.
constexpr int kBinThreads = 256;
constexpr int kBinItems = 8;

__global__ void __launch_bounds__(kBinThreads)
tile_bins_kernel(const uint32_t* __restrict__ keys, int64_t count, int32_t tile_n_bits,
                 int32_t num_tiles, int64_t num_bins, int2* bins, unsigned* err) {
  pdl_enter();
  const int64_t base =
      (static_cast<int64_t>(blockIdx.x) * kBinThreads + threadIdx.x) * kBinItems;
  const int lane = threadIdx.x & 31;
  uint32_t k[kBinItems];
  if (base + kBinItems <= count) {
    const uint4 a = *reinterpret_cast<const uint4*>(keys + base);
    const uint4 b = *reinterpret_cast<const uint4*>(keys + base + 4);
    k[0] = a.x; k[1] = a.y; k[2] = a.z; k[3] = a.w;
    k[4] = b.x; k[5] = b.y; k[6] = b.z; k[7] = b.w;
  } else {
#pragma unroll
    for (int m = 0; m < kBinItems; ++m) k[m] = base + m < count ? keys[base + m] : 0u;
  }
  uint32_t prev_key = __shfl_up_sync(0xffffffffu, k[kBinItems - 1], 1);
  if (lane == 0 && base > 0 && base - 1 < count) prev_key = keys[base - 1];
  const uint32_t mask = (1u << tile_n_bits) - 1u;
#pragma unroll
  for (int m = 0; m < kBinItems; ++m) {
    const int64_t idx = base + m;
    const uint32_t key = k[m];
    const uint32_t pk = m == 0 ? prev_key : k[m - 1];
    if (idx >= count) break;
    const int64_t cur = static_cast<int64_t>(key >> tile_n_bits) * num_tiles + (key & mask);
    if (cur >= num_bins) {
      atomicOr(err, kErrBinRange);
      continue;
    }
    if (idx == 0) {
      bins[cur].x = 0;
      continue;
    }
    if (idx == count - 1) bins[cur].y = static_cast<int32_t>(count);
    const int64_t prev = static_cast<int64_t>(pk >> tile_n_bits) * num_tiles + (pk & mask);
    if (prev != cur && prev < num_bins) {
      bins[prev].y = static_cast<int32_t>(idx);
      bins[cur].x = static_cast<int32_t>(idx);
    }
  }
}

template <typename K, int ITEMS, int NT, bool FILTER, int RB>
void set_onesweep_smem() {
  static bool done = false;  // per instantiation: static + dynamic exceeds 48 KiB
  if (!done) {
    cudaFuncSetAttribute(onesweep_kernel<K, ITEMS, NT, FILTER, RB>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(NT * ITEMS * (sizeof(K) + sizeof(int32_t))));
    done = true;
  }
}

// Stable LSD sort of `count` keys by their low `bits` bits in RB-bit digits. With
// s.filter_sentinel the all-ones keys are dropped by the histogram and the first pass, s.vcount
// receives how many keys remain, and the later passes read that device-side count (their grids
// stay sized for `count`; surplus tiles leave).
template <typename K, int ITEMS, int NT, int RB>
int sort_impl(const SortScratch& s, int64_t count, int bits, cudaStream_t stream) {
  constexpr int D = 1 << RB;
  const int passes = (bits + RB - 1) / RB;
  uint32_t* hist = s.hist;
  uint32_t* offsets = s.hist + kRadixHistWords;
  constexpr int TILE = NT * ITEMS;
  const int64_t tiles = (count + TILE - 1) / TILE;
  const int64_t rows = tiles * D;  // look-back words of one pass
  // Small sorts: passes alternate between two halves of the look-back words; the first is
  // cleared here with the histograms and tile tickets, and each pass clears the half its
  // predecessor used, which its successor reuses, so no launch sits between the passes (the
  // depth sort of 8M pairs 0.250 -> 0.240 ms, a one-image bin sort 0.146 -> 0.142). Large
  // sorts (look-back words above kSelfClearBytes) memset each pass's words right before it:
  // cleared a pass ahead, or by the clear kernel, the bin sort of eight 1080p images took
  // 0.976-0.981 ms instead of 0.955.
  const bool halves = passes > 1 && s.status_words >= 2 * rows &&
                      rows * sizeof(unsigned long long) <= kSelfClearBytes;
  unsigned long long* half[2] = {s.status, halves ? s.status + rows : s.status};
  {
    const ClearSpan spans[3] = {{hist, sizeof(uint32_t) * kRadixHistWords},
                                {s.tile_counters, sizeof(int) * 8},
                                {s.status, halves ? sizeof(unsigned long long) * rows : 0}};
    launch_clear(spans, 3, stream);
  }
  const int64_t hblocks = (count + kHistThreads * kHistItems - 1) / (kHistThreads * kHistItems);
  launch_pdl(radix_hist_kernel<K, RB>, static_cast<unsigned>(hblocks), kHistThreads, 0, stream,
      reinterpret_cast<const K*>(s.keys[0]), count, s.filter_sentinel, passes, hist);
  launch_pdl(radix_scan_kernel<D>, passes, D, 0, stream, hist, offsets,
      s.filter_sentinel ? s.vcount : nullptr);
  const size_t smem = TILE * (sizeof(K) + sizeof(int32_t));
  set_onesweep_smem<K, ITEMS, NT, false, RB>();
  set_onesweep_smem<K, ITEMS, NT, true, RB>();
  int cur = 0;
  for (int p = 0; p < passes; ++p) {
    unsigned long long* status = half[p & 1];
    unsigned long long* clear_next = halves && p + 1 < passes ? half[(p + 1) & 1] : nullptr;
    if (!halves) cudaMemsetAsync(status, 0, sizeof(unsigned long long) * rows, stream);
    const K* kin = reinterpret_cast<const K*>(s.keys[cur]);
    K* kout = reinterpret_cast<K*>(s.keys[cur ^ 1]);
    if (s.filter_sentinel && p == 0)
      launch_pdl(onesweep_kernel<K, ITEMS, NT, true, RB>, static_cast<unsigned>(tiles), NT, smem,
          stream, kin, s.vals[cur], kout, s.vals[cur ^ 1], count, nullptr, RB * p, offsets + p * D,
          status, s.tile_counters + p, s.err, clear_next);
    else
      launch_pdl(onesweep_kernel<K, ITEMS, NT, false, RB>, static_cast<unsigned>(tiles), NT, smem,
          stream, kin, s.vals[cur], kout, s.vals[cur ^ 1], count,
          s.filter_sentinel ? s.vcount : nullptr, RB * p, offsets + p * D, status,
          s.tile_counters + p, s.err, clear_next);
    cur ^= 1;
  }
  return cur;
}

// 9-bit digits where they save a pass (17-18, 25-27 and 33-36 significant bits), else 8.
int radix_digit_bits(int bits) {
  const int p8 = (bits + 7) / 8, p9 = (bits + 8) / 9;
  return p9 < p8 && p9 <= kRadixHistWords / 512 ? 9 : 8;
}

}  // namespace

void launch_clear(const ClearSpan* spans, int count, cudaStream_t stream) {
  ClearArgs a = {};
  int64_t vec = 0;
  auto flush = [&]() {
    if (a.count == 0) return;
    // a few 16-byte stores per thread, at most 8 CTAs per SM's worth of the grid
    const int64_t want = (vec + 4 * kClearThreads - 1) / (4 * kClearThreads);
    const unsigned blocks =
        static_cast<unsigned>(std::min<int64_t>(std::max<int64_t>(want, 1), 148 * 8));
    launch_pdl(clear_kernel, blocks, kClearThreads, 0, stream, a);
    a = ClearArgs{};
    vec = 0;
  };
  for (int i = 0; i < count; ++i) {
    if (spans[i].p == nullptr || spans[i].bytes == 0) continue;
    if (reinterpret_cast<uintptr_t>(spans[i].p) % 4 != 0 || spans[i].bytes % 4 != 0) {
      cudaMemsetAsync(spans[i].p, 0, spans[i].bytes, stream);  // not whole words: no kernel
      continue;
    }
    a.p[a.count] = static_cast<uint32_t*>(spans[i].p);
    a.words[a.count] = static_cast<int64_t>(spans[i].bytes / 4);
    vec = std::max<int64_t>(vec, a.words[a.count] / 4 + 1);
    if (++a.count == kClearMaxSpans) flush();
  }
  flush();
}

void launch_depth_minmax(const float* depths, const int32_t* radii, int64_t total, int64_t n,
                         int32_t B, int32_t* depth_mm, cudaStream_t stream) {
  launch_pdl(seed_minmax_kernel, static_cast<unsigned>((B + 127) / 128), 128, 0, stream, depth_mm,
      B);
  if (total <= 0) return;
  // the vector path needs 16-byte aligned runs (cudaMalloc'd operands; checked) and n >= 16
  const bool aligned = (reinterpret_cast<uintptr_t>(depths) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(radii) % 16 == 0);
  if (aligned && n >= kMmItems) {
    const int64_t blocks = (total + kMmThreads * kMmItems - 1) / (kMmThreads * kMmItems);
    launch_pdl(depth_minmax_kernel, static_cast<unsigned>(blocks), kMmThreads, 0, stream, depths,
        radii, total, n, depth_mm);
  } else {
    const int64_t blocks = (total + kMmThreads - 1) / kMmThreads;
    launch_pdl(depth_minmax_small_n_kernel, static_cast<unsigned>(blocks), kMmThreads, 0, stream,
        depths, radii, total, n, depth_mm);
  }
}

void launch_depth_span(const int32_t* depth_mm, int32_t B, unsigned* span_out,
                       cudaStream_t stream) {
  launch_pdl(depth_span_kernel, 1, 256, 0, stream, depth_mm, B, span_out);
}

void launch_pair_keys(const PairKeyArgs& a, bool key64, void* keys, int32_t* vals,
                      cudaStream_t stream) {
  const int64_t blocks = (a.total + kPrepThreads - 1) / kPrepThreads;
  if (blocks == 0) return;
  if (key64)
    launch_pdl(pair_prep_kernel<uint64_t>, static_cast<unsigned>(blocks), kPrepThreads, 0, stream,
        a, static_cast<uint64_t*>(keys), vals);
  else
    launch_pdl(pair_prep_kernel<uint32_t>, static_cast<unsigned>(blocks), kPrepThreads, 0, stream,
        a, static_cast<uint32_t*>(keys), vals);
}

int64_t sorted_offsets_tiles(int64_t total) {
  return (total + kScanThreads * kScanItems - 1) / (kScanThreads * kScanItems);
}

void launch_sorted_offsets(const int32_t* perm, const int32_t* counts, int64_t total,
                           const int32_t* dtotal, int32_t* offsets, unsigned long long* status,
                           int* ticket, unsigned* err, cudaStream_t stream) {
  const int64_t tiles = sorted_offsets_tiles(total);
  if (tiles == 0) return;
  const ClearSpan spans[2] = {{ticket, sizeof(int)}, {status, sizeof(unsigned long long) * tiles}};
  launch_clear(spans, 2, stream);
  launch_pdl(sorted_offsets_kernel, static_cast<unsigned>(tiles), kScanThreads, 0, stream, perm,
      counts, total, dtotal, offsets, status, ticket, err);
}

void launch_emit(const EmitArgs& a, cudaStream_t stream) {
  const int64_t blocks = (a.total + kEmitThreads - 1) / kEmitThreads;  // 32 pairs per warp
  if (blocks == 0) return;
  launch_pdl(emit_sorted_kernel, static_cast<unsigned>(blocks), kEmitThreads, 0, stream, a);
}

void launch_reference_keys(const uint32_t* bin_keys, const int32_t* gids, int64_t count,
                           const PairKeyArgs& a, int64_t* out, cudaStream_t stream) {
  const int64_t blocks = (count + 255) / 256;
  if (blocks == 0) return;
  launch_pdl(reference_keys_kernel, static_cast<unsigned>(blocks), 256, 0, stream, bin_keys, gids,
      count, a, out);
}

int sort_tile_items(bool key64) { return kSortThreads * (key64 ? kItems64 : kItems32); }

int radix_sort_pairs(const SortScratch& s, bool key64, int64_t count, int bits,
                     cudaStream_t stream) {
  if (s.filter_sentinel && count <= 0) {
    cudaMemsetAsync(s.vcount, 0, sizeof(int32_t), stream);
    return 0;
  }
  // with the filter even a single key goes through, so that vcount is written
  if (count <= 1 && !s.filter_sentinel) return 0;
  if (radix_digit_bits(bits) == 9)
    return key64 ? sort_impl<uint64_t, kItems64, kSortThreads, 9>(s, count, bits, stream)
                 : sort_impl<uint32_t, kItems32, kSortThreads, 9>(s, count, bits, stream);
  return key64 ? sort_impl<uint64_t, kItems64, kSortThreads, 8>(s, count, bits, stream)
               : sort_impl<uint32_t, kItems32, kSortThreads, 8>(s, count, bits, stream);
}

int radix_passes(int bits) {
  const int rb = radix_digit_bits(bits);
  return (bits + rb - 1) / rb;
}

void launch_tile_bins(const uint32_t* keys, int64_t count, int32_t tile_n_bits,
                      int32_t num_tiles, int64_t num_bins, int32_t* tile_bins, unsigned* err,
                      cudaStream_t stream) {
  const int64_t per_block = static_cast<int64_t>(kBinThreads) * kBinItems;
  const int64_t blocks = (count + per_block - 1) / per_block;
  if (blocks == 0) return;
  launch_pdl(tile_bins_kernel, static_cast<unsigned>(blocks), kBinThreads, 0, stream, keys, count,
      tile_n_bits, num_tiles, num_bins, reinterpret_cast<int2*>(tile_bins), err);
}
}  // namespace splax
