// Fused mean-squared-error loss of a rendered image stack and its gradient: the objective of
// the benchmark configurations 1 and 2 (sum((img - target)^2) / denom), taken in one pass
// over both arrays instead of separate difference, square, sum and scale passes.
//
// Forward: a fixed grid of CTAs, each thread summing its grid-stride share (16-byte vector
// loads when both arrays are 16-byte aligned) in fp32, a block reduction, one fp64 partial
// per CTA, and the last CTA to finish adding the partials in index order -- so the result is
// deterministic. Backward: grad = v_loss * 2 (img - target) / denom, with v_loss read from
// device memory (no host synchronisation).
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

constexpr int kLossThreads = 256;
// grid strides per loop trip in both kernels, their loads issued together: the config-2 pair
// (995 MB: two 199 MB arrays read by each kernel, the gradient written) went from 0.187 to
// 0.180 ms per step, 0.85 of the measured HBM copy rate
constexpr int kLossUnroll = 4;

__device__ __forceinline__ float sq_diff_sum(float4 a, float4 b) {
  const float dx = a.x - b.x, dy = a.y - b.y, dz = a.z - b.z, dw = a.w - b.w;
  return fmaf(dx, dx, fmaf(dy, dy, fmaf(dz, dz, dw * dw)));
}

__global__ void __launch_bounds__(kLossThreads)
mse_loss_kernel(const float* __restrict__ img, const float* __restrict__ tgt, int64_t count,
                bool vec, double inv_denom, double* partials, unsigned* done, float* loss) {
  pdl_enter();
  float acc = 0.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLossThreads;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kLossThreads + threadIdx.x;
  int64_t tail = 0;
  if (vec) {
    const int64_t n4 = count / 4;
    const float4* a4 = reinterpret_cast<const float4*>(img);
    const float4* b4 = reinterpret_cast<const float4*>(tgt);
    // kLossUnroll grid strides per trip: their loads are issued together (bytes in flight)
    float part[kLossUnroll];
#pragma unroll
    for (int u = 0; u < kLossUnroll; ++u) part[u] = 0.0f;
    int64_t i = t0;
    for (; i + (kLossUnroll - 1) * stride < n4; i += kLossUnroll * stride) {
      float4 a[kLossUnroll], b[kLossUnroll];
#pragma unroll
      for (int u = 0; u < kLossUnroll; ++u) {
        a[u] = __ldcs(a4 + i + u * stride);
        b[u] = __ldcs(b4 + i + u * stride);
      }
#pragma unroll
      for (int u = 0; u < kLossUnroll; ++u) part[u] += sq_diff_sum(a[u], b[u]);
    }
    for (; i < n4; i += stride) part[0] += sq_diff_sum(__ldcs(a4 + i), __ldcs(b4 + i));
#pragma unroll
    for (int u = 0; u < kLossUnroll; ++u) acc += part[u];
    tail = n4 * 4;
  }
  for (int64_t i = tail + t0; i < count; i += stride) {
    const float d = img[i] - tgt[i];
    acc = fmaf(d, d, acc);
  }
  __shared__ float s_warp[kLossThreads / 32];
  __shared__ bool s_last;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_warp[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int w = 0; w < kLossThreads / 32; ++w) b += s_warp[w];
    partials[blockIdx.x] = b;
    __threadfence();
    s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    double total = 0.0;
    for (unsigned b = 0; b < gridDim.x; ++b) total += *(volatile double*)(partials + b);
    *loss = static_cast<float>(total * inv_denom);
    *done = 0u;  // ready for the next call on this stream
  }
}

__global__ void __launch_bounds__(kLossThreads)
mse_loss_bwd_kernel(const float* __restrict__ img, const float* __restrict__ tgt, int64_t count,
                    bool vec, float scale, const float* __restrict__ v_loss,
                    float* __restrict__ grad) {
  pdl_enter();
  const float s = scale * *v_loss;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLossThreads;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kLossThreads + threadIdx.x;
  int64_t tail = 0;
  if (vec) {
    const int64_t n4 = count / 4;
    const float4* a4 = reinterpret_cast<const float4*>(img);
    const float4* b4 = reinterpret_cast<const float4*>(tgt);
    float4* g4 = reinterpret_cast<float4*>(grad);
    auto diff = [s](float4 a, float4 b) {
      return make_float4(s * (a.x - b.x), s * (a.y - b.y), s * (a.z - b.z), s * (a.w - b.w));
    };
    int64_t i = t0;
    for (; i + (kLossUnroll - 1) * stride < n4; i += kLossUnroll * stride) {
      float4 a[kLossUnroll], b[kLossUnroll];
#pragma unroll
      for (int u = 0; u < kLossUnroll; ++u) {
        a[u] = __ldcs(a4 + i + u * stride);
        b[u] = __ldcs(b4 + i + u * stride);
      }
#pragma unroll
      for (int u = 0; u < kLossUnroll; ++u) __stcs(g4 + i + u * stride, diff(a[u], b[u]));
    }
    for (; i < n4; i += stride) __stcs(g4 + i, diff(__ldcs(a4 + i), __ldcs(b4 + i)));
    tail = n4 * 4;
  }
  for (int64_t i = tail + t0; i < count; i += stride) grad[i] = s * (img[i] - tgt[i]);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int mse_loss_blocks() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return 4 * sms;
}

void launch_mse_loss(const float* img, const float* tgt, int64_t count, double inv_denom,
                     double* partials, unsigned* done, float* loss, int blocks,
                     cudaStream_t stream) {
  const bool vec = aligned16(img) && aligned16(tgt);
  launch_pdl(mse_loss_kernel, blocks, kLossThreads, 0, stream, img, tgt, count, vec, inv_denom,
      partials, done, loss);
}

void launch_mse_loss_bwd(const float* img, const float* tgt, int64_t count, float scale,
                         const float* v_loss, float* grad, int blocks, cudaStream_t stream) {
  const bool vec = aligned16(img) && aligned16(tgt) && aligned16(grad);
  launch_pdl(mse_loss_bwd_kernel, blocks, kLossThreads, 0, stream, img, tgt, count, vec, scale,
      v_loss, grad);
}

}  // namespace splax
