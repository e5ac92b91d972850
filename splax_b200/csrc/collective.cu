// Sum all-reduce of the fp32 gaussian gradients across the ranks of a camera-sharded step,
// through NVLink SHARP (NVLS) on the NVSwitch fabric. The reference has no multi-device path;
// the exchange it stands for is the psum of the 14 per-gaussian gradient floats (means 3,
// scales 3, quats 4, colors 3, opacity 1) that a shard_map over cameras would lower to an NCCL
// all-reduce.
//
// The gradient buffer is a symmetric allocation: every rank holds a copy at the same offset,
// and one multicast address covers all copies. Rank r owns the r-th shard of the buffer's
// 16-byte vectors. For each vector of its shard it issues one multimem.ld_reduce (the switch
// reads the vector from every rank and returns the sum) and one multimem.st of the sum (the
// switch writes it to every rank's copy). Each GPU's NVLink then carries its whole buffer once
// out (the reads of all shards) and once in (the multicast stores): 2 x 4 x n bytes whatever
// the rank count, with no local reduction pass.
//
// The step runs as three launches on the caller's stream: an entry barrier (every rank's
// gradients are complete), the shard reduction, an exit barrier (every shard's sums have
// landed everywhere). The barriers exchange epoch numbers through a flag array that lives in
// each rank's copy of the buffer: rank r stores the epoch into slot r of every peer's array
// (plain peer stores, release at system scope) and waits until its own array holds the epoch
// in every slot (acquire loads). Waits are bounded; on expiry the kernel sets an error bit and
// returns. Once a wait has given up, the error word stays set and every later launch of the
// exchange on this rank (barriers, reductions) returns before touching peer or multicast memory:
// a rank that failed to meet its peers stops issuing NVLink traffic toward them, so memory of a
// rank that has left is never read or written through the switch afterwards.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

constexpr int kMaxRanks = 8;
constexpr long long kBarrierSpinLimit = 1ll << 24;  // polls with a 64 ns back-off: seconds
constexpr int kReduceThreads = 512;
constexpr int kReduceUnroll = 1;  // 4 and 8 loads in flight per thread measured no faster

struct PeerFlags {
  unsigned long long* p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The rank's own error word (local memory); nonzero once a barrier of this or an earlier call
// gave up.
__device__ __forceinline__ bool exchange_failed(const unsigned* err) {
  return *reinterpret_cast<const volatile unsigned*>(err) != 0u;
}

// Lane q < world signals peer q and then waits for peer q's signal.
__global__ void __launch_bounds__(32)
nvls_barrier_kernel(PeerFlags peers, int rank, int world, unsigned long long epoch,
                    unsigned* err) {
  const int q = threadIdx.x;
  if (q >= world || exchange_failed(err)) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  st_release_sys(peers.p[q] + rank, epoch);
  const unsigned long long* mine = peers.p[rank] + q;
  long long spins = 0;
  while (ld_acquire_sys(mine) < epoch) {
    if (++spins > kBarrierSpinLimit) {
      atomicOr(err, kErrBarrierTimeout);
      break;
    }
    __nanosleep(64);
  }
}

__device__ __forceinline__ float4 mm_ld_reduce(const float* a) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(a)
               : "memory");
  return r;
}
__device__ __forceinline__ void mm_st(float* a, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Each thread keeps kReduceUnroll loads in flight (consecutive threads, consecutive vectors).
__global__ void __launch_bounds__(kReduceThreads)
nvls_reduce_kernel(float* mc, int64_t n, int rank, int world, const unsigned* err) {
  if (exchange_failed(err)) return;  // the entry barrier did not meet every rank
  const int64_t nv = n >> 2;
  const int64_t per = (nv + world - 1) / world;
  const int64_t v0 = min(nv, static_cast<int64_t>(rank) * per);
  const int64_t v1 = min(nv, v0 + per);
  constexpr int64_t kChunk = static_cast<int64_t>(kReduceThreads) * kReduceUnroll;
  for (int64_t c = v0 + static_cast<int64_t>(blockIdx.x) * kChunk; c < v1;
       c += static_cast<int64_t>(gridDim.x) * kChunk) {
    float4 r[kReduceUnroll];
#pragma unroll
    for (int u = 0; u < kReduceUnroll; ++u) {
      const int64_t v = c + u * kReduceThreads + threadIdx.x;
      if (v < v1) r[u] = mm_ld_reduce(mc + 4 * v);
    }
#pragma unroll
    for (int u = 0; u < kReduceUnroll; ++u) {
      const int64_t v = c + u * kReduceThreads + threadIdx.x;
      if (v < v1) mm_st(mc + 4 * v, r[u]);
    }
  }
  // the n % 4 trailing floats: the last rank, first block
  if (rank == world - 1 && blockIdx.x == 0) {
    const int64_t i = 4 * nv + threadIdx.x;
    if (i < n) {
      float x;
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];"
                   : "=f"(x)
                   : "l"(mc + i)
                   : "memory");
      asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc + i), "f"(x)
                   : "memory");
    }
  }
  // this thread's multicast stores are performed system-wide before the kernel retires, so the
  // exit barrier's release store (next launch) follows them
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// The training step's exchange and optimiser in one pass: for each 16-byte vector of this rank's
// shard, the switch sums the gradients of every rank (multimem.ld_reduce), the rank applies Adam
// with its shard of the moments (the optimiser state is sharded over the ranks), and multicasts
// the updated parameters into every rank's copy (multimem.st). Reduce-scatter, update and
// parameter all-gather in one kernel, moving the bytes of one all-reduce. Element e's learning
// rate is the rate of the parameter group whose [start, end) holds e.
__device__ __forceinline__ float group_lr(const NvlsAdamGroups& gr, int64_t e) {
  float lr = gr.lr[0];
#pragma unroll
  for (int k = 1; k < kAdamMaxSegs; ++k)
    if (k < gr.count && e >= gr.end[k - 1]) lr = gr.lr[k];
  return lr;
}

__global__ void __launch_bounds__(kReduceThreads)
nvls_adam_kernel(const float* grad_mc, float* param_mc, const float* __restrict__ param_local,
                 float* __restrict__ m_shard, float* __restrict__ v_shard, int64_t n, int rank,
                 int world, NvlsAdamGroups gr, float b1, float b2, float bc1, float bc2,
                 float eps, const unsigned* err) {
  if (exchange_failed(err)) return;  // the entry barrier did not meet every rank
  const int64_t nv = n >> 2;
  const int64_t per = (nv + world - 1) / world;
  const int64_t v0 = min(nv, static_cast<int64_t>(rank) * per);
  const int64_t v1 = min(nv, v0 + per);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kReduceThreads;
  for (int64_t v = v0 + static_cast<int64_t>(blockIdx.x) * kReduceThreads + threadIdx.x; v < v1;
       v += stride) {
    const float4 g = mm_ld_reduce(grad_mc + 4 * v);
    float4 p = *reinterpret_cast<const float4*>(param_local + 4 * v);
    float4 m = reinterpret_cast<float4*>(m_shard)[v - v0];
    float4 w = reinterpret_cast<float4*>(v_shard)[v - v0];
    const int64_t e = 4 * v;
    adam_one(p.x, g.x, m.x, w.x, group_lr(gr, e), b1, b2, bc1, bc2, eps);
    adam_one(p.y, g.y, m.y, w.y, group_lr(gr, e + 1), b1, b2, bc1, bc2, eps);
    adam_one(p.z, g.z, m.z, w.z, group_lr(gr, e + 2), b1, b2, bc1, bc2, eps);
    adam_one(p.w, g.w, m.w, w.w, group_lr(gr, e + 3), b1, b2, bc1, bc2, eps);
    reinterpret_cast<float4*>(m_shard)[v - v0] = m;
    reinterpret_cast<float4*>(v_shard)[v - v0] = w;
    mm_st(param_mc + 4 * v, p);
  }
  // the n % 4 trailing elements: the last rank, first block; their moments follow its shard's
  if (rank == world - 1 && blockIdx.x == 0) {
    const int64_t i = 4 * nv + threadIdx.x;
    if (i < n) {
      float g;
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];"
                   : "=f"(g)
                   : "l"(grad_mc + i)
                   : "memory");
      float p = param_local[i];
      const int64_t j = 4 * (v1 - v0) + (i - 4 * nv);
      adam_one(p, g, m_shard[j], v_shard[j], group_lr(gr, i), b1, b2, bc1, bc2, eps);
      asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(param_mc + i), "f"(p)
                   : "memory");
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

}  // namespace

int launch_nvls_barrier(unsigned long long* const* flags, int rank, int world,
                        unsigned long long epoch, unsigned* err, cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return -1;
  PeerFlags pf{};
  for (int q = 0; q < world; ++q) {
    if (flags[q] == nullptr) return -1;
    pf.p[q] = flags[q];
  }
  nvls_barrier_kernel<<<1, 32, 0, stream>>>(pf, rank, world, epoch, err);
  return 0;
}

int64_t nvls_adam_shard_len(int64_t n, int rank, int world) {
  const int64_t nv = n >> 2;
  const int64_t per = (nv + world - 1) / world;
  const int64_t v0 = std::min(nv, static_cast<int64_t>(rank) * per);
  const int64_t v1 = std::min(nv, v0 + per);
  return 4 * (v1 - v0) + (rank == world - 1 ? n - 4 * nv : 0);
}

int launch_nvls_adam(const float* grad_mc, float* param_mc, const float* param_local,
                     float* m_shard, float* v_shard, int64_t n, int rank, int world,
                     const NvlsAdamGroups& gr, float b1, float b2, float bc1, float bc2, float eps,
                     const unsigned* err, cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || n < 0) return -1;
  if (n == 0) return 0;
  if ((reinterpret_cast<uintptr_t>(grad_mc) | reinterpret_cast<uintptr_t>(param_mc) |
       reinterpret_cast<uintptr_t>(param_local) | reinterpret_cast<uintptr_t>(m_shard) |
       reinterpret_cast<uintptr_t>(v_shard)) % 16 != 0)
    return -1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per = ((n >> 2) + world - 1) / world;
  int64_t blocks = (per + kReduceThreads - 1) / kReduceThreads;
  blocks = blocks < 1 ? 1 : (blocks > 4 * sms ? 4 * sms : blocks);
  nvls_adam_kernel<<<static_cast<unsigned>(blocks), kReduceThreads, 0, stream>>>(
      grad_mc, param_mc, param_local, m_shard, v_shard, n, rank, world, gr, b1, b2, bc1, bc2,
      eps, err);
  return 0;
}

int launch_nvls_allreduce(float* multicast, int64_t n, int rank, int world, const unsigned* err,
                          cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || n < 0) return -1;
  if (n == 0 || world == 1) return 0;
  if (reinterpret_cast<uintptr_t>(multicast) % 16 != 0) return -1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per = ((n >> 2) + world - 1) / world;
  const int64_t chunk = static_cast<int64_t>(kReduceThreads) * kReduceUnroll;
  int64_t blocks = (per + chunk - 1) / chunk;
  blocks = blocks < 1 ? 1 : (blocks > 4 * sms ? 4 * sms : blocks);
  nvls_reduce_kernel<<<static_cast<unsigned>(blocks), kReduceThreads, 0, stream>>>(
      multicast, n, rank, world, err);
  return 0;
}

}  // namespace splax
