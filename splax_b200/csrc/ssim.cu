// Fused photometric loss of the batched training step (config 3): (1 - lambda) L1 + lambda
// D-SSIM against targets, for a stack of B RGB images (B, H, W, 3), as taken by the
// reference's make_step (scripts/train_colmap.py:202-221: l1 = mean |img - gt| per view,
// dssim = 1 - ssim(img, gt) per view, both averaged over the views).
//
// SSIM follows its published definition (Wang et al. 2004) in the form the reference calls
// (dm_pix.ssim defaults): an 11-tap Gaussian window of sigma 1.5 applied separably with VALID
// extent, so the map covers (H-10) x (W-10) x 3 entries; mu / sigma statistics of a, b, a^2,
// b^2, ab; variances clamped below at eps_f32^2, the covariance clamped in magnitude to
// sqrt(var_a var_b); k1 = 0.01, k2 = 0.03, max_val = 1.
//
// The partial loss of the views given is
//   (1 - lambda) sum|a - b| / (V H W 3) + lambda (B / V - sum ssim_map / (V (H-10)(W-10) 3)),
// with V the total number of views over all ranks, so per-rank partials add up to the
// reference's loss and each rank's gradient is already the global one.
//
// Forward: one CTA per 32 x 16 map tile and image; the RGB input tile with its 10-pixel halo is
// staged in shared memory, the horizontal then vertical window sums of the five statistics
// produce the map, and each CTA writes fp64 partial sums (SSIM map, and L1 over the input
// pixels it owns). A single-block pass adds the partials in index order (deterministic).
// Backward (recompute): one CTA per 32 x 16 input tile; it recomputes the statistics on the
// map region its pixels feed (halo 10), forms per map entry the sensitivities of SSIM to mu_a,
// E[a^2] and E[ab] (through the clamps), and applies the adjoint window:
//   dL/da = -s (W*G_mu + 2 a W*G_aa + b W*G_ab) + l1 sign(a - b),
// s and l1 the SSIM and L1 coefficients of the loss above, times the incoming cotangent.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace splax {
namespace {

constexpr int kWin = 11;          // window taps
constexpr int kHalo = kWin - 1;   // 10
constexpr int kTileX = 32, kTileY = 16;
constexpr int kSsimThreads = 256;
constexpr float kC1 = 0.0001f;    // (0.01 * 1)^2
constexpr float kC2 = 0.0009f;    // (0.03 * 1)^2
constexpr float kVarFloor = 1.4210854715202004e-14f;  // FLT_EPSILON^2

__constant__ float c_win[kWin];

// SSIM entry from the window statistics (E[a], E[b], E[a^2], E[b^2], E[ab]) with the clamps;
// optionally its sensitivities to E[a] (total, through the variances), E[a^2] and E[ab].
template <bool GRAD>
__device__ __forceinline__ float ssim_entry(float ea, float eb, float eaa, float ebb, float eab,
                                            float* g_mu, float* g_aa, float* g_ab) {
  const float mu00 = ea * ea, mu11 = eb * eb, mu01 = ea * eb;
  const float r00 = eaa - mu00, r11 = ebb - mu11, r01 = eab - mu01;
  const float s00 = fmaxf(kVarFloor, r00), s11 = fmaxf(kVarFloor, r11);
  const float lim = sqrtf(s00 * s11);
  const float mag = fabsf(r01);
  const float sg = r01 > 0.0f ? 1.0f : (r01 < 0.0f ? -1.0f : 0.0f);
  const bool clamp01 = !(mag < lim);  // |r01| >= sqrt(s00 s11): the bound is taken
  const float s01 = sg * fminf(lim, mag);
  const float A = 2.0f * mu01 + kC1, Bn = 2.0f * s01 + kC2;
  const float Cd = mu00 + mu11 + kC1, Dd = s00 + s11 + kC2;
  const float N = A * Bn, D = Cd * Dd;
  const float S = N / D;
  if constexpr (GRAD) {
    // dS/d(mu0) at fixed sigmas, dS/d(s00), dS/d(s01)
    const float dS_mu0 = 2.0f * eb * Bn / D - S * 2.0f * ea / Cd;
    float dS_s00 = -S / Dd;
    const float dS_s01 = 2.0f * A / D;
    float d_r01 = 0.0f;
    if (clamp01) {
      // s01 = sg * sqrt(s00 s11): flows into s00 (s11 has no gradient)
      if (lim > 0.0f) dS_s00 += dS_s01 * sg * 0.5f * s11 / lim;
    } else {
      d_r01 = dS_s01 * sg * sg;  // d(sg * |r01|)/d r01 = sg^2
    }
    const float d_r00 = r00 > kVarFloor ? dS_s00 : 0.0f;
    // r00 = E[a^2] - mu0^2, r01 = E[ab] - mu0 mu1
    *g_aa = d_r00;
    *g_ab = d_r01;
    *g_mu = dS_mu0 - 2.0f * ea * d_r00 - eb * d_r01;
  }
  return S;
}

__device__ __forceinline__ float sgn(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

// ------------------------------------------------------------------ forward
// Map tile [mx0, mx0+32) x [my0, my0+16) needs input [mx0, mx0+42) x [my0, my0+26).
constexpr int kInX = kTileX + kHalo, kInY = kTileY + kHalo;  // 42 x 26

__global__ void __launch_bounds__(kSsimThreads)
l1_dssim_fwd_kernel(const float* __restrict__ img, const float* __restrict__ tgt, int32_t H,
                    int32_t W, int32_t tiles_x, double2* partials) {
  __shared__ float s_a[3][kInY][kInX];
  __shared__ float s_b[3][kInY][kInX];
  __shared__ float s_h[5][kInY][kTileX];  // horizontal window sums of one channel
  __shared__ double s_red[2][kSsimThreads / 32];
  const int tx = blockIdx.x % tiles_x, ty = blockIdx.x / tiles_x;
  const int64_t b = blockIdx.y;
  const int Hm = H - kHalo, Wm = W - kHalo;
  const int mx0 = tx * kTileX, my0 = ty * kTileY;
  const float* ia = img + b * H * static_cast<int64_t>(W) * 3;
  const float* ib = tgt + b * H * static_cast<int64_t>(W) * 3;
  // L1 ownership: input pixels [my0, my0+16) x [mx0, mx0+32); the last tile row / column also
  // owns the 10 pixels beyond the map
  const int ox1 = (tx == tiles_x - 1) ? W : mx0 + kTileX;
  const int oy1 = (ty == static_cast<int>(gridDim.x) / tiles_x - 1) ? H : my0 + kTileY;
  float l1 = 0.0f;
  for (int i = threadIdx.x; i < kInY * kInX * 3; i += kSsimThreads) {
    const int c = i % 3, px = (i / 3) % kInX, py = i / (3 * kInX);
    const int gx = mx0 + px, gy = my0 + py;
    float va = 0.0f, vb = 0.0f;
    if (gx < W && gy < H) {
      const int64_t o = (static_cast<int64_t>(gy) * W + gx) * 3 + c;
      va = ia[o];
      vb = ib[o];
      if (gx < ox1 && gy < oy1) l1 += fabsf(va - vb);
    }
    s_a[c][py][px] = va;
    s_b[c][py][px] = vb;
  }
  __syncthreads();
  float ssum = 0.0f;
  for (int c = 0; c < 3; ++c) {
    for (int i = threadIdx.x; i < kInY * kTileX; i += kSsimThreads) {
      const int y = i / kTileX, x = i % kTileX;
      float h0 = 0.f, h1 = 0.f, h2 = 0.f, h3 = 0.f, h4 = 0.f;
#pragma unroll
      for (int u = 0; u < kWin; ++u) {
        const float w = c_win[u], a = s_a[c][y][x + u], bb = s_b[c][y][x + u];
        h0 = fmaf(w, a, h0);
        h1 = fmaf(w, bb, h1);
        h2 = fmaf(w, a * a, h2);
        h3 = fmaf(w, bb * bb, h3);
        h4 = fmaf(w, a * bb, h4);
      }
      s_h[0][y][x] = h0; s_h[1][y][x] = h1; s_h[2][y][x] = h2; s_h[3][y][x] = h3;
      s_h[4][y][x] = h4;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kTileY * kTileX; i += kSsimThreads) {
      const int y = i / kTileX, x = i % kTileX;
      if (my0 + y >= Hm || mx0 + x >= Wm) continue;
      float e[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int v = 0; v < kWin; ++v) {
        const float w = c_win[v];
#pragma unroll
        for (int q = 0; q < 5; ++q) e[q] = fmaf(w, s_h[q][y + v][x], e[q]);
      }
      ssum += ssim_entry<false>(e[0], e[1], e[2], e[3], e[4], nullptr, nullptr, nullptr);
    }
    __syncthreads();
  }
  double ds = ssum, dl = l1;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    ds += __shfl_xor_sync(0xffffffffu, ds, off);
    dl += __shfl_xor_sync(0xffffffffu, dl, off);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { s_red[0][warp] = ds; s_red[1][warp] = dl; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, l = 0.0;
    for (int w = 0; w < kSsimThreads / 32; ++w) { a += s_red[0][w]; l += s_red[1][w]; }
    partials[blockIdx.y * gridDim.x + blockIdx.x] = make_double2(a, l);
  }
}

__global__ void l1_dssim_finalize_kernel(const double2* partials, int64_t count, double l1_scale,
                                         double ssim_scale, double ssim_const, float* loss) {
  __shared__ double s_a[256], s_l[256];
  double a = 0.0, l = 0.0;
  for (int64_t i = threadIdx.x; i < count; i += 256) {  // fixed assignment and order
    a += partials[i].x;
    l += partials[i].y;
  }
  s_a[threadIdx.x] = a;
  s_l[threadIdx.x] = l;
  __syncthreads();
  for (int st = 128; st > 0; st >>= 1) {
    if (threadIdx.x < st) {
      s_a[threadIdx.x] += s_a[threadIdx.x + st];
      s_l[threadIdx.x] += s_l[threadIdx.x + st];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0)
    *loss = static_cast<float>(l1_scale * s_l[0] + ssim_const - ssim_scale * s_a[0]);
}

// ------------------------------------------------------------------ backward
// Input tile [x0, x0+32) x [y0, y0+16); the map entries feeding it are [x0-10, x0+32) x
// [y0-10, y0+16), whose statistics need input [x0-10, x0+42) x [y0-10, y0+26).
constexpr int kBx = kTileX + 2 * kHalo, kBy = kTileY + 2 * kHalo;  // 52 x 36 input
constexpr int kMx = kTileX + kHalo, kMy = kTileY + kHalo;          // 42 x 26 map

// FUSED (the loss and its gradient in one pass, for a unit cotangent): the CTA also sums the
// SSIM map entries it owns ([x0, x0+32) x [y0, y0+16) of the map) and the L1 of its input
// pixels, and writes them as its fp64 partials.
template <bool FUSED>
__global__ void __launch_bounds__(kSsimThreads)
l1_dssim_bwd_kernel(const float* __restrict__ img, const float* __restrict__ tgt, int32_t H,
                    int32_t W, int32_t tiles_x, float l1_scale, float ssim_grad_scale,
                    const float* __restrict__ v_loss, float* __restrict__ grad,
                    double2* partials) {
  extern __shared__ float smem[];
  float* s_a = smem;                    // [kBy][kBx]
  float* s_b = s_a + kBy * kBx;         // [kBy][kBx]
  float* s_h = s_b + kBy * kBx;         // [5][kBy][kMx] horizontal sums
  float* s_g = s_h + 5 * kBy * kMx;     // [3][kMy][kMx] sensitivities
  float* s_gh = s_g + 3 * kMy * kMx;    // [3][kMy][kTileX] adjoint horizontal sums
  const int tx = blockIdx.x % tiles_x, ty = blockIdx.x / tiles_x;
  const int64_t b = blockIdx.y;
  const int Hm = H - kHalo, Wm = W - kHalo;
  const int x0 = tx * kTileX, y0 = ty * kTileY;
  const int bx0 = x0 - kHalo, by0 = y0 - kHalo;  // input origin of the staged region
  const float* ia = img + b * H * static_cast<int64_t>(W) * 3;
  const float* ib = tgt + b * H * static_cast<int64_t>(W) * 3;
  float* go = grad + b * H * static_cast<int64_t>(W) * 3;
  const float vl = FUSED ? 1.0f : *v_loss;
  const float s_ssim = ssim_grad_scale * vl, s_l1 = l1_scale * vl;
  float ssum = 0.0f, l1 = 0.0f;  // FUSED: owned map entries and input pixels
  for (int c = 0; c < 3; ++c) {
    for (int i = threadIdx.x; i < kBy * kBx; i += kSsimThreads) {
      const int py = i / kBx, px = i % kBx;
      const int gx = bx0 + px, gy = by0 + py;
      float va = 0.0f, vb = 0.0f;
      if (gx >= 0 && gy >= 0 && gx < W && gy < H) {
        const int64_t o = (static_cast<int64_t>(gy) * W + gx) * 3 + c;
        va = ia[o];
        vb = ib[o];
      }
      s_a[i] = va;
      s_b[i] = vb;
    }
    __syncthreads();
    // horizontal window sums for map columns [x0-10, x0+32) on every staged row
    for (int i = threadIdx.x; i < kBy * kMx; i += kSsimThreads) {
      const int y = i / kMx, x = i % kMx;
      float h[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int u = 0; u < kWin; ++u) {
        const float w = c_win[u], a = s_a[y * kBx + x + u], bb = s_b[y * kBx + x + u];
        h[0] = fmaf(w, a, h[0]);
        h[1] = fmaf(w, bb, h[1]);
        h[2] = fmaf(w, a * a, h[2]);
        h[3] = fmaf(w, bb * bb, h[3]);
        h[4] = fmaf(w, a * bb, h[4]);
      }
#pragma unroll
      for (int q = 0; q < 5; ++q) s_h[(q * kBy + y) * kMx + x] = h[q];
    }
    __syncthreads();
    // sensitivities of each map entry (zero outside the map)
    for (int i = threadIdx.x; i < kMy * kMx; i += kSsimThreads) {
      const int y = i / kMx, x = i % kMx;
      const int my = by0 + y, mx = bx0 + x;
      float gm = 0.0f, gaa = 0.0f, gab = 0.0f;
      if (my >= 0 && mx >= 0 && my < Hm && mx < Wm) {
        float e[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int v = 0; v < kWin; ++v) {
          const float w = c_win[v];
#pragma unroll
          for (int q = 0; q < 5; ++q) e[q] = fmaf(w, s_h[(q * kBy + y + v) * kMx + x], e[q]);
        }
        const float S = ssim_entry<true>(e[0], e[1], e[2], e[3], e[4], &gm, &gaa, &gab);
        if (FUSED && y >= kHalo && x >= kHalo) ssum += S;
      }
      s_g[(0 * kMy + y) * kMx + x] = gm;
      s_g[(1 * kMy + y) * kMx + x] = gaa;
      s_g[(2 * kMy + y) * kMx + x] = gab;
    }
    __syncthreads();
    // adjoint window, horizontal: input column x0+x receives map columns x0+x-10 .. x0+x,
    // staged at x .. x+10 (window tap u = 10 - (staged offset))
    for (int i = threadIdx.x; i < kMy * kTileX; i += kSsimThreads) {
      const int y = i / kTileX, x = i % kTileX;
      float h[3] = {0.f, 0.f, 0.f};
#pragma unroll
      for (int u = 0; u < kWin; ++u) {
        const float w = c_win[kHalo - u];
#pragma unroll
        for (int q = 0; q < 3; ++q) h[q] = fmaf(w, s_g[(q * kMy + y) * kMx + x + u], h[q]);
      }
#pragma unroll
      for (int q = 0; q < 3; ++q) s_gh[(q * kMy + y) * kTileX + x] = h[q];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kTileY * kTileX; i += kSsimThreads) {
      const int y = i / kTileX, x = i % kTileX;
      const int gy = y0 + y, gx = x0 + x;
      if (gy >= H || gx >= W) continue;
      float g[3] = {0.f, 0.f, 0.f};
#pragma unroll
      for (int v = 0; v < kWin; ++v) {
        const float w = c_win[kHalo - v];
#pragma unroll
        for (int q = 0; q < 3; ++q) g[q] = fmaf(w, s_gh[(q * kMy + y + v) * kTileX + x], g[q]);
      }
      const float a = s_a[(y + kHalo) * kBx + x + kHalo], bb = s_b[(y + kHalo) * kBx + x + kHalo];
      const float d_ssim = g[0] + 2.0f * a * g[1] + bb * g[2];
      go[(static_cast<int64_t>(gy) * W + gx) * 3 + c] = s_ssim * d_ssim + s_l1 * sgn(a - bb);
      if (FUSED) l1 += fabsf(a - bb);
    }
    __syncthreads();
  }
  if constexpr (FUSED) {
    __shared__ double s_red[2][kSsimThreads / 32];
    double ds = ssum, dl = l1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      ds += __shfl_xor_sync(0xffffffffu, ds, off);
      dl += __shfl_xor_sync(0xffffffffu, dl, off);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
      s_red[0][warp] = ds;
      s_red[1][warp] = dl;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double sa = 0.0, sl = 0.0;
      for (int w = 0; w < kSsimThreads / 32; ++w) {
        sa += s_red[0][w];
        sl += s_red[1][w];
      }
      partials[blockIdx.y * gridDim.x + blockIdx.x] = make_double2(sa, sl);
    }
  }
}

constexpr size_t kBwdSmem =
    sizeof(float) * (2 * kBy * kBx + 5 * kBy * kMx + 3 * kMy * kMx + 3 * kMy * kTileX);

}  // namespace

void ssim_set_window(const float* w11) {
  cudaMemcpyToSymbol(c_win, w11, sizeof(float) * kWin);
}

int64_t l1_dssim_partials(int32_t B, int32_t H, int32_t W) {
  const int Hm = H - kHalo, Wm = W - kHalo;
  const int64_t tiles = static_cast<int64_t>((Wm + kTileX - 1) / kTileX) *
                        ((Hm + kTileY - 1) / kTileY);
  return tiles * B;
}

// partials of the fused pass: one per input tile and image
static int64_t l1_dssim_grad_partials(int32_t B, int32_t H, int32_t W) {
  return static_cast<int64_t>((W + kTileX - 1) / kTileX) * ((H + kTileY - 1) / kTileY) * B;
}

int64_t l1_dssim_partials_max(int32_t B, int32_t H, int32_t W) {
  const int64_t a = l1_dssim_partials(B, H, W), b = l1_dssim_grad_partials(B, H, W);
  return a > b ? a : b;
}

void launch_l1_dssim(const float* img, const float* tgt, int32_t B, int32_t H, int32_t W,
                     double l1_scale, double ssim_scale, double ssim_const, double2* partials,
                     float* loss, cudaStream_t stream) {
  const int Hm = H - kHalo, Wm = W - kHalo;
  const int tiles_x = (Wm + kTileX - 1) / kTileX, tiles_y = (Hm + kTileY - 1) / kTileY;
  dim3 grid(tiles_x * tiles_y, B);
  l1_dssim_fwd_kernel<<<grid, kSsimThreads, 0, stream>>>(img, tgt, H, W, tiles_x, partials);
  l1_dssim_finalize_kernel<<<1, 256, 0, stream>>>(partials, l1_dssim_partials(B, H, W), l1_scale,
                                                  ssim_scale, ssim_const, loss);
}

void launch_l1_dssim_bwd(const float* img, const float* tgt, int32_t B, int32_t H, int32_t W,
                         float l1_scale, float ssim_grad_scale, const float* v_loss, float* grad,
                         cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(l1_dssim_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kBwdSmem));
    attr = true;
  }
  const int tiles_x = (W + kTileX - 1) / kTileX, tiles_y = (H + kTileY - 1) / kTileY;
  dim3 grid(tiles_x * tiles_y, B);
  l1_dssim_bwd_kernel<false><<<grid, kSsimThreads, kBwdSmem, stream>>>(
      img, tgt, H, W, tiles_x, l1_scale, ssim_grad_scale, v_loss, grad, nullptr);
}

void launch_l1_dssim_and_grad(const float* img, const float* tgt, int32_t B, int32_t H,
                              int32_t W, double l1_scale, double ssim_scale, double ssim_const,
                              float l1_grad_scale, float ssim_grad_scale, double2* partials,
                              float* loss, float* grad, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(l1_dssim_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kBwdSmem));
    attr = true;
  }
  const int tiles_x = (W + kTileX - 1) / kTileX, tiles_y = (H + kTileY - 1) / kTileY;
  dim3 grid(tiles_x * tiles_y, B);
  l1_dssim_bwd_kernel<true><<<grid, kSsimThreads, kBwdSmem, stream>>>(
      img, tgt, H, W, tiles_x, l1_grad_scale, ssim_grad_scale, nullptr, grad, partials);
  l1_dssim_finalize_kernel<<<1, 256, 0, stream>>>(partials, l1_dssim_grad_partials(B, H, W),
                                                  l1_scale, ssim_scale, ssim_const, loss);
}

}  // namespace splax
