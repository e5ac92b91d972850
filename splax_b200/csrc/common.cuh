// Shared device helpers of the splax_b200 kernels: constants, the deterministic logarithm,
// saturating float->int truncation and the opacity-aware ellipse tile walk.
//
// Files that produce integer outputs (project.cu, sort.cu) are compiled with --fmad=false and
// IEEE division / square root, so every float operation below rounds exactly as written and
// the tile counts, radii and keys are bit-identical to the C oracle's restatement.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace splax {

// splax/_intersect.py:17-20, splax/_rasterize/_kernels.py:188-192
constexpr int kBlockWidth = 16;            // 16x16 pixel tiles
constexpr int kBlockSize = 256;            // pixels per tile
constexpr float kGaussianExtendSq = static_cast<float>(3.33 * 3.33);  // rounded to fp32
constexpr float kAlphaThreshold = 1.0f / 255.0f;
constexpr float kAlphaMax = 0.999f;
constexpr float kTransmittanceMin = 1e-4f;

// Device error word bits (read back by the host after a launch sequence).
constexpr unsigned kErrLookbackTimeout = 1u << 0;  // a bounded spin-wait gave up
constexpr unsigned kErrEmitCount = 1u << 1;        // emission disagreed with cum_tiles_hit
constexpr unsigned kErrNegativeDepthKey = 1u << 2; // 64-bit key of a negative depth
constexpr unsigned kErrCountOverflow = 1u << 3;    // intersections exceed int32
constexpr unsigned kErrBinRange = 1u << 4;         // a sorted key decoded outside B*T bins
constexpr unsigned kErrBarrierTimeout = 1u << 5;   // a cross-rank barrier wait gave up

constexpr long long kSpinLimit = 1ll << 24;  // iterations before a look-back wait gives up

__device__ __forceinline__ int32_t f2i(float x) {
  // cvt.rzi.s32.f32: truncation, saturating, NaN -> 0 (what wp.int32(x) does on the GPU)
  return static_cast<int32_t>(x);
}
__device__ __forceinline__ float fmin_w(float a, float b) { return a < b ? a : b; }
__device__ __forceinline__ float fmax_w(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ int32_t imin(int32_t a, int32_t b) { return a < b ? a : b; }
__device__ __forceinline__ int32_t imax(int32_t a, int32_t b) { return a > b ? a : b; }

// Natural logarithm: atanh series log(m) = 2 atanh((m-1)/(m+1)) (Abramowitz & Stegun
// 4.1.27) on m in [sqrt(1/2), sqrt(2)), Cody-Waite split of ln 2 for the exponent. Written as
// plain IEEE operations in a fixed order so the integer tile walk it feeds is reproducible
// on any IEEE fp32 host.
__device__ __forceinline__ float splat_logf(float x) {
  if (!(x > 0.0f)) return x == 0.0f ? -__int_as_float(0x7f800000) : __int_as_float(0x7fc00000);
  if (x == __int_as_float(0x7f800000)) return x;
  int32_t e = 0;
  uint32_t bits = __float_as_uint(x);
  if (bits < 0x00800000u) {
    x = __fmul_rn(x, 8388608.0f);
    bits = __float_as_uint(x);
    e = -23;
  }
  e += static_cast<int32_t>(bits >> 23) - 127;
  float m = __uint_as_float((bits & 0x007fffffu) | 0x3f800000u);
  if (m > 1.41421356f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  float s2 = __fmul_rn(s, s);
  float p = 0.0909090936f;
  p = __fadd_rn(__fmul_rn(p, s2), 0.111111112f);
  p = __fadd_rn(__fmul_rn(p, s2), 0.142857149f);
  p = __fadd_rn(__fmul_rn(p, s2), 0.200000003f);
  p = __fadd_rn(__fmul_rn(p, s2), 0.333333343f);
  p = __fadd_rn(__fmul_rn(p, s2), 1.0f);
  float fe = static_cast<float>(e);
  float lm = __fmul_rn(__fmul_rn(2.0f, s), p);
  return __fadd_rn(__fmul_rn(fe, 0.693145751953125f),
                   __fadd_rn(lm, __fmul_rn(fe, 1.42860677e-06f)));
}

// Opacity-aware isocontour level t = min(3.33^2, 2 ln(opac / (1/255))),
// splax/_project/_kernels.py:227.
__device__ __forceinline__ float iso_level(float opac) {
  return fmin_w(kGaussianExtendSq, 2.0f * splat_logf(opac / kAlphaThreshold));
}

// Tight ellipse and its tile walk state (splax/_intersect.py:23-107). Component 0 of the
// bbox / rect pairs is the walk's outer axis.
struct Ellipse {
  float A, B, C, disc, t, px, py;
  float bmin0, bmin1, bmax0, bmax1, amin1, amax1;
  int32_t rmin0, rmin1, rmax0, rmax1;
  bool valid, isY;
};

__device__ __forceinline__ void ellipse_init(float A, float B, float C, float t, float px,
                                             float py, int32_t tile_w, int32_t tile_h,
                                             Ellipse& s) {
  s.valid = false;
  s.isY = false;
  s.A = A; s.B = B; s.C = C; s.t = t; s.px = px; s.py = py;
  float disc = B * B - A * C;
  s.disc = disc;
  float nt = -t / disc;
  float x_ext = sqrtf(nt * C);
  float y_ext = sqrtf(nt * A);
  float bminx = px - x_ext, bminy = py - y_ext;
  float bmaxx = px + x_ext, bmaxy = py + y_ext;
  float bxc = B * x_ext / C;
  float bya = B * y_ext / A;
  float aminx = py + bxc, aminy = px + bya;  // bbox_argmin = (py + Bx/C, px + By/A)
  float amaxx = py - bxc, amaxy = px - bya;
  const float ts = static_cast<float>(kBlockWidth);
  int32_t rminx = imax(0, imin(tile_w, f2i(bminx / ts)));
  int32_t rminy = imax(0, imin(tile_h, f2i(bminy / ts)));
  int32_t rmaxx = imax(0, imin(tile_w, f2i(bmaxx / ts + 1.0f)));
  int32_t rmaxy = imax(0, imin(tile_h, f2i(bmaxy / ts + 1.0f)));
  int32_t xs = rmaxx - rminx, ys = rmaxy - rminy;
  if (ys * xs == 0) return;
  bool isY = ys < xs;
  s.isY = isY;
  if (isY) {
    s.rmin0 = rminy; s.rmin1 = rminx; s.rmax0 = rmaxy; s.rmax1 = rmaxx;
    s.bmin0 = bminy; s.bmin1 = bminx; s.bmax0 = bmaxy; s.bmax1 = bmaxx;
    s.amin1 = aminx; s.amax1 = amaxx;
  } else {
    s.rmin0 = rminx; s.rmin1 = rminy; s.rmax0 = rmaxx; s.rmax1 = rmaxy;
    s.bmin0 = bminx; s.bmin1 = bminy; s.bmax0 = bmaxx; s.bmax1 = bmaxy;
    s.amin1 = aminy; s.amax1 = amaxy;
  }
  s.valid = true;
}

// Cross-axis extent of the ellipse at one line of the outer axis (splax/_intersect.py:110-133):
// the interval [lo, hi] on the line `coord`, from the ellipse fields (pu / pv: the centre along
// the outer / cross axis, coeff: the outer axis' quadratic coefficient). The one definition the
// sequential and the warp-cooperative walks share.
__device__ __forceinline__ void walk_intersect(float B, float disc, float t, float coeff, float pu,
                                               float pv, float coord, float& lo, float& hi) {
  float h = coord - pu;
  float sq = sqrtf(disc * h * h + t * coeff);
  float bh = (-B) * h;
  lo = (bh - sq) / coeff + pv;
  hi = (bh + sq) / coeff + pv;
}

__device__ __forceinline__ void ellipse_intersect(const Ellipse& s, float coord, float& lo,
                                                  float& hi) {
  walk_intersect(s.B, s.disc, s.t, s.isY ? s.A : s.C, s.isY ? s.py : s.px, s.isY ? s.px : s.py,
                 coord, lo, hi);
}

// Leading line of the walk (splax/_intersect.py:136-143)
__device__ __forceinline__ void ellipse_init_span(const Ellipse& s, float& i0, float& i1) {
  float line0 = static_cast<float>(s.rmin0) * static_cast<float>(kBlockWidth);
  if (s.bmin0 <= line0) {
    ellipse_intersect(s, line0, i0, i1);
    return;
  }
  i0 = s.bmax1;
  i1 = s.bmin1;
}

// One outer column: [mn, mx) cross-axis tiles; rolls the intersect pair (splax/_intersect.py:
// 146-169).
__device__ __forceinline__ void ellipse_column(int32_t u, const Ellipse& s, float& i0,
                                               float& i1, int32_t& mn, int32_t& mx) {
  const float block = static_cast<float>(kBlockWidth);
  float min_line = static_cast<float>(u) * block;
  float max_line = min_line + block;
  float j0 = i0, j1 = i1;
  if (max_line <= s.bmax0) ellipse_intersect(s, max_line, j0, j1);
  float emin = (min_line <= s.amin1 && s.amin1 < max_line) ? s.bmin1 : fmin_w(i0, j0);
  float emax = (min_line <= s.amax1 && s.amax1 < max_line) ? s.bmax1 : fmax_w(i1, j1);
  mn = imax(s.rmin1, imin(s.rmax1, f2i(emin / block)));
  mx = imin(s.rmax1, imax(s.rmin1, f2i(emax / block + 1.0f)));
  i0 = j0;
  i1 = j1;
}

__device__ __forceinline__ int32_t ellipse_tile_count(const Ellipse& s) {
  if (!s.valid) return 0;
  float i0, i1;
  ellipse_init_span(s, i0, i1);
  int32_t count = 0;
  for (int32_t u = s.rmin0; u < s.rmax0; ++u) {
    int32_t mn, mx;
    ellipse_column(u, s, i0, i1, mn, mx);
    count += mx - mn;
  }
  return count;
}

// ---------------------------------------------------------------- warp-cooperative walk
// The ellipse walks of the 32 pairs of a warp (one pair per lane), taken row by row with one
// row per lane instead of one pair per lane: a warp's cost follows the rows of its 32 pairs,
// not its largest pair. A row is one outer-axis tile line u of a pair's walk. Its start state is
// the walk's rolling intersect pair at the row's lower line, computed directly from its
// definition (the intersect at the last line <= bmax0 above rmin0, or the initial span); its end
// state is the next row's start state, taken from the next lane by shuffle when that lane holds
// the same pair's next row. Every float operation is the sequential walk's (ellipse_column), so
// [mn, mx) is bit-identical to it.

// Largest lane whose (non-decreasing across lanes) v is <= key.
__device__ __forceinline__ int lift_find(int v, int key) {
  int pos = 0;
#pragma unroll
  for (int st = 16; st > 0; st >>= 1) {
    const int c = __shfl_sync(0xffffffffu, v, pos + st);
    if (c <= key) pos += st;
  }
  return pos;
}

struct WarpWalk {
  // per lane: B, disc, t, coeff, pu, pv, bmax0, amin1, amax1, bmin1, bmax1, i0, i1
  float f[13][32];
  // per lane: rmin0, rmin1, rmax1, isY, first row (exclusive scan of the row counts)
  int32_t n[5][32];
};

// Shares this lane's walk (e.valid false: no rows). Returns the warp's row count; rexc = this
// lane's first row. Ends with __syncwarp.
__device__ __forceinline__ int warp_walk_share(WarpWalk& w, int lane, const Ellipse& e,
                                               int& rexc) {
  float i0 = 0.0f, i1 = 0.0f;
  int R = 0;
  if (e.valid) {
    ellipse_init_span(e, i0, i1);
    R = e.rmax0 > e.rmin0 ? e.rmax0 - e.rmin0 : 0;
  }
  int rinc = R;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, rinc, o);
    if (lane >= o) rinc += v;
  }
  rexc = rinc - R;
  w.f[0][lane] = e.B;
  w.f[1][lane] = e.disc;
  w.f[2][lane] = e.t;
  w.f[3][lane] = e.isY ? e.A : e.C;
  w.f[4][lane] = e.isY ? e.py : e.px;
  w.f[5][lane] = e.isY ? e.px : e.py;
  w.f[6][lane] = e.bmax0;
  w.f[7][lane] = e.amin1;
  w.f[8][lane] = e.amax1;
  w.f[9][lane] = e.bmin1;
  w.f[10][lane] = e.bmax1;
  w.f[11][lane] = i0;
  w.f[12][lane] = i1;
  w.n[0][lane] = e.rmin0;
  w.n[1][lane] = e.rmin1;
  w.n[2][lane] = e.rmax1;
  w.n[3][lane] = e.isY ? 1 : 0;
  w.n[4][lane] = rexc;
  __syncwarp();
  return __shfl_sync(0xffffffffu, rinc, 31);
}

// Row r of the shared walk (all 32 lanes call together; rows = the warp's row count, rexc = this
// lane's warp_walk_share value). For r < rows: ow = the pair's lane, u = the outer line, [mn, mx)
// = ellipse_column's cross-axis range. For r >= rows: mn = mx = 0.
__device__ __forceinline__ void warp_walk_row(const WarpWalk& w, int lane, int rexc, int r,
                                              int rows, int& ow, int& u, int32_t& mn,
                                              int32_t& mx) {
  const bool has = r < rows;
  ow = lift_find(rexc, has ? r : rows);
  const float B = w.f[0][ow], disc = w.f[1][ow], t = w.f[2][ow];
  const float coeff = w.f[3][ow], pu = w.f[4][ow], pv = w.f[5][ow];
  const float bmax0 = w.f[6][ow], amin1 = w.f[7][ow], amax1 = w.f[8][ow];
  const float bmin1 = w.f[9][ow], bmax1 = w.f[10][ow];
  const int32_t rmin0 = w.n[0][ow], rmin1 = w.n[1][ow], rmax1 = w.n[2][ow];
  u = rmin0 + (r - w.n[4][ow]);
  float s0 = w.f[11][ow], s1 = w.f[12][ow];
  if (has && u > rmin0) {
    int m = u;  // the last line (m * 16, the previous row's upper line) the walk intersected
    while (m > rmin0 && !(static_cast<float>(m - 1) * 16.0f + 16.0f <= bmax0)) --m;
    if (m > rmin0)
      walk_intersect(B, disc, t, coeff, pu, pv, static_cast<float>(m - 1) * 16.0f + 16.0f, s0,
                     s1);
  }
  const float n0 = __shfl_down_sync(0xffffffffu, s0, 1);
  const float n1 = __shfl_down_sync(0xffffffffu, s1, 1);
  const int now = __shfl_down_sync(0xffffffffu, ow, 1);
  const bool next_same = lane < 31 && r + 1 < rows && now == ow;
  const float min_line = static_cast<float>(u) * 16.0f;
  const float max_line = min_line + 16.0f;
  float j0 = s0, j1 = s1;
  if (next_same) {
    j0 = n0;
    j1 = n1;
  } else if (has && max_line <= bmax0) {
    walk_intersect(B, disc, t, coeff, pu, pv, max_line, j0, j1);
  }
  mn = 0;
  mx = 0;
  if (has) {
    const float emin = (min_line <= amin1 && amin1 < max_line) ? bmin1 : fmin_w(s0, j0);
    const float emax = (min_line <= amax1 && amax1 < max_line) ? bmax1 : fmax_w(s1, j1);
    mn = imax(rmin1, imin(rmax1, f2i(emin / 16.0f)));
    mx = imin(rmax1, imax(rmin1, f2i(emax / 16.0f + 1.0f)));
  }
}

// One Adam update in optax's scale_by_adam form (fp32): m = (1 - b1) g + b1 m,
// v = (1 - b2) g^2 + b2 v, p += -lr (m / bc1) / (sqrt(v / bc2) + eps), bc = 1 - b^step. Shared
// by the single-GPU update and the fused NVLS exchange-and-update, so both round alike.
__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, float lr,
                                         float b1, float b2, float bc1, float bc2, float eps) {
  m = (1.0f - b1) * g + b1 * m;
  v = (1.0f - b2) * (g * g) + b2 * v;
  const float mh = m / bc1, vh = v / bc2;
  p = p + (-lr) * (mh / (sqrtf(vh) + eps));
}

// Programmatic dependent launch (sm_90+). Every kernel of the path starts with pdl_enter():
// griddepcontrol.wait returns once the stream predecessor has completed and its writes are
// visible (at once for a launch without the attribute), so nothing is read early; then
// launch_dependents lets the successor's CTAs be scheduled as soon as every CTA of this grid
// has started, which hides the successor's launch and ramp behind this grid's last wave.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Hardware base-2 exponential (MUFU): the blend kernels' exponent is pre-scaled by log2(e).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// -infinity: log2 of a zero opacity, the staged exponent offset of a transparent record
__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// Packed fp32x2 arithmetic (sm_100 FFMA2 / FMUL2 / FADD2): two lanes of IEEE round-to-nearest
// math per instruction, each lane bit-identical to the scalar fmaf / * / +.
__device__ __forceinline__ float2 splat2(float s) { return make_float2(s, s); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
// 1 - a, rounded once (fma(a, -1, 1) is the exact difference rounded like 1.0f - a)
__device__ __forceinline__ float2 one_minus2(float2 a) {
  return __ffma2_rn(a, make_float2(-1.0f, -1.0f), make_float2(1.0f, 1.0f));
}

// log2(e) / 2 and log2(e), the scales of the staged conic q = -(log2 e / 2) * (a, 2b, c)
constexpr float kHalfLog2e = 0.721347520444482f;
constexpr float kLog2e = 1.442695040888963f;

// Ordered-integer image of a float, so atomicMin / atomicMax on int32 order like floats.
__device__ __forceinline__ int32_t float_to_ordered(float f) {
  int32_t i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float ordered_to_float(int32_t i) {
  return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff);
}

// Relaxed gpu-scope accesses for look-back status words: the flag and the value share one
// 64-bit word, so a reader that sees the flag sees its value and no fence is needed.
__device__ __forceinline__ void st_relaxed(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Decoupled look-back by one full warp over single-word tile states (2-bit flag: 1 aggregate,
// 2 inclusive prefix, in the top bits; value below): the 32 lanes read 32 predecessors per
// round trip, sum up to the nearest inclusive one, and repeat further back if there is none.
// Returns the exclusive prefix of `tile`. Spins are bounded; on expiry sets kErrLookbackTimeout.
constexpr unsigned long long kLookbackAgg = 1ull << 62;
constexpr unsigned long long kLookbackInc = 2ull << 62;
constexpr unsigned long long kLookbackMask = (1ull << 62) - 1;

__device__ __forceinline__ long long warp_lookback(const unsigned long long* status, int64_t tile,
                                                   unsigned* err) {
  constexpr unsigned long long kInc = kLookbackInc, kMask = kLookbackMask;
  const int lane = threadIdx.x & 31;
  long long prefix = 0;
  int64_t base = tile - 1;
  long long spins = 0;
  while (base >= 0) {
    const int64_t j = base - lane;
    const unsigned long long s = j >= 0 ? ld_relaxed(status + j) : kInc;  // before tile 0: 0
    const unsigned long long flag = s & ~kMask;
    const unsigned inc = __ballot_sync(0xffffffffu, flag == kInc);
    const unsigned notready = __ballot_sync(0xffffffffu, flag == 0);
    const int first = inc ? __ffs(inc) - 1 : 31;
    const unsigned needed = first == 31 ? 0xffffffffu : ((2u << first) - 1u);
    if (notready & needed) {
      if (++spins > kSpinLimit) {
        if (lane == 0) atomicOr(err, kErrLookbackTimeout);
        break;
      }
      continue;
    }
    long long v = lane <= first ? static_cast<long long>(s & kMask) : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    prefix += v;
    if (inc) break;
    base -= 32;
  }
  return prefix;
}

// Release / acquire accesses for look-back status words.
__device__ __forceinline__ void st_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Warp reduce-scatter of K per-lane values: after the call, every lane whose return value c
// is >= 0 and whose lane bit 0 is clear holds in v[0] the warp-wide sum of component c (each
// component has exactly one such holder). A butterfly that halves the slot count at every
// exchange, so K values cost about K shuffles instead of 5K for K full reductions.
template <int K, int OFF>
struct ReduceScatter {
  static __device__ __forceinline__ void run(float* v, int lane, int& comp, int& real) {
    if constexpr (K == 1) {
#pragma unroll
      for (int off = OFF; off > 0; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    } else {
      constexpr int H = (K + 1) / 2;
      const bool bit = (lane & OFF) != 0;
#pragma unroll
      for (int j = 0; j < H; ++j) {
        float lo = v[j];
        float hi = (j + H < K) ? v[j + H] : 0.0f;
        float recv = __shfl_xor_sync(0xffffffffu, bit ? lo : hi, OFF);
        v[j] = (bit ? hi : lo) + recv;
      }
      if (bit) {
        comp += H;
        real = real - H;
      } else {
        real = real < H ? real : H;
      }
      ReduceScatter<H, OFF / 2>::run(v, lane, comp, real);
    }
  }
};

template <int K>
__device__ __forceinline__ int warp_reduce_scatter(float (&v)[K], int lane) {
  static_assert(K >= 1 && K <= 32, "1..32 components");
  int comp = 0, real = K;
  ReduceScatter<K, 16>::run(v, lane, comp, real);
  return (real >= 1 && (lane & 1) == 0) ? comp : -1;
}

}  // namespace splax
