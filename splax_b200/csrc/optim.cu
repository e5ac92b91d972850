// Fused per-parameter Adam update of the batched training step (config 3; the reference builds
// it with optax.adam per parameter group, scripts/train_colmap.py:639-645). One launch updates
// up to kAdamMaxSegs parameter arrays in place, each with its own learning rate, following
// optax's scale_by_adam (optax 0.2.8): m = (1 - b1) g + b1 m, v = (1 - b2) g^2 + b2 v,
// m_hat = m / (1 - b1^t), v_hat = v / (1 - b2^t), p += -lr m_hat / (sqrt(v_hat) + eps), in fp32.
// Elementwise and HBM-bound: 4 floats read and 3 written per parameter, 16-byte accesses when
// a segment is 16-byte aligned.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

constexpr int kAdamThreads = 256;

__global__ void __launch_bounds__(kAdamThreads) adam_kernel(AdamSegs s, float b1, float b2,
                                                            float bc1, float bc2, float eps) {
  const AdamSeg& seg = s.seg[blockIdx.y];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kAdamThreads;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kAdamThreads + threadIdx.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(seg.p) | reinterpret_cast<uintptr_t>(seg.g) |
                     reinterpret_cast<uintptr_t>(seg.m) | reinterpret_cast<uintptr_t>(seg.v)) &
                    15u) == 0;
  int64_t tail = 0;
  if (vec) {
    const int64_t n4 = seg.n / 4;
    float4* p4 = reinterpret_cast<float4*>(seg.p);
    const float4* g4 = reinterpret_cast<const float4*>(seg.g);
    float4* m4 = reinterpret_cast<float4*>(seg.m);
    float4* v4 = reinterpret_cast<float4*>(seg.v);
    for (int64_t i = t0; i < n4; i += stride) {
      float4 p = p4[i], m = m4[i], v = v4[i];
      const float4 g = g4[i];
      adam_one(p.x, g.x, m.x, v.x, seg.lr, b1, b2, bc1, bc2, eps);
      adam_one(p.y, g.y, m.y, v.y, seg.lr, b1, b2, bc1, bc2, eps);
      adam_one(p.z, g.z, m.z, v.z, seg.lr, b1, b2, bc1, bc2, eps);
      adam_one(p.w, g.w, m.w, v.w, seg.lr, b1, b2, bc1, bc2, eps);
      p4[i] = p;
      m4[i] = m;
      v4[i] = v;
    }
    tail = n4 * 4;
  }
  for (int64_t i = tail + t0; i < seg.n; i += stride)
    adam_one(seg.p[i], seg.g[i], seg.m[i], seg.v[i], seg.lr, b1, b2, bc1, bc2, eps);
}

}  // namespace

void launch_adam(const AdamSegs& s, int32_t count, float b1, float b2, float bc1, float bc2,
                 float eps, cudaStream_t stream) {
  if (count <= 0) return;
  int64_t biggest = 0;
  for (int k = 0; k < count; ++k) biggest = s.seg[k].n > biggest ? s.seg[k].n : biggest;
  if (biggest == 0) return;
  const int64_t want = (biggest / 4 + kAdamThreads - 1) / kAdamThreads;
  const unsigned gx = static_cast<unsigned>(want < 1 ? 1 : (want > 2048 ? 2048 : want));
  adam_kernel<<<dim3(gx, count), kAdamThreads, 0, stream>>>(s, b1, b2, bc1, bc2, eps);
}

}  // namespace splax
