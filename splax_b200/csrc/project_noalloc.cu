// splax_project_noalloc: the projection forward for callers that must not allocate device
// memory.
//
// splax_project keeps its scan's look-back words in scratch the library allocates with
// cudaMalloc on first use. Some callers cannot let a library do that: an XLA custom call in a
// JAX process whose allocator has preallocated most of the GPU (cudaMalloc then fails or
// fragments what is left), or an embedder whose memory budget is fixed up front. This entry
// point runs the
// same kernel with its scratch in a file-scope __device__ array instead, so it never calls
// cudaMalloc, cudaFree or any allocating routine. The caller still passes every input and
// output buffer.
//
// Limits and rules:
//  - at most kNoAllocMaxPairs = 16,777,216 (camera, gaussian) pairs per call (B * n); larger
//    calls are rejected with SPLAX_ERR_INVALID_ARGUMENT. The array is 128 KiB + 16 bytes
//    (16,386 eight-byte words) and every GPU that loads the library holds it until the process
//    exits;
//  - the first call on each device resolves the array's device address (cudaGetSymbolAddress,
//    with that device current); make that first call before any stream capture;
//  - every call shares the one array and rewrites it (the scan words are cleared at the start
//    of each call), so calls that overlap on the GPU -- two streams at once -- race and must be
//    serialised by the caller;
//  - the call's device error word (int32 overflow of the intersection count, a look-back wait
//    that gave up) is the array's word 1, which no other entry point reads: it is read back,
//    and reported, only when SPLAX_SYNC_CHECK=1. Without it those errors go unreported here.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "../../include/splax_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

constexpr int64_t kNoAllocMaxPairs = int64_t(1) << 24;
constexpr int64_t kNoAllocTiles = kNoAllocMaxPairs / kProjScanTile;
// word 0: block ticket, word 1: device error word, words 2..: one look-back word per scan tile
constexpr int64_t kNoAllocWords = kNoAllocTiles + 2;

static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocWords];
static_assert(sizeof(g_noalloc_scratch) == 128 * 1024 + 16,
              "the documented size of the no-alloc scratch is 128 KiB + 16 bytes");

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned long long* g_noalloc_ptr[kMaxDevices] = {};

}  // namespace
}  // namespace splax

using namespace splax;

extern "C" int splax_project_noalloc(
    const float* means3d, int64_t means3d_rows, const float* scales, int64_t scales_rows,
    const float* quats_xyzw, int64_t quats_rows, const float* viewmat, int64_t viewmat_rows,
    const float* opacities, int64_t opacities_rows, const float* gaussian_transforms,
    int64_t transforms_rows, const int32_t* transform_ids, int32_t num_gaussians,
    int32_t num_transforms, int32_t has_transforms, int32_t img_h, int32_t img_w, float fx,
    float fy, float cx, float cy, float glob_scale, float clip_thresh, int64_t total, float* xys,
    float* depths, int32_t* radii, float* conics, int32_t* num_tiles_hit,
    int32_t* cum_tiles_hit, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t n = num_gaussians;
  if (n <= 0 || total <= 0 || total % n != 0 || img_h <= 0 || img_w <= 0)
    return record_error(SPLAX_ERR_INVALID_ARGUMENT,
                        "project_noalloc: invalid num_gaussians, total or image size");
  if (total > kNoAllocMaxPairs) {
    char msg[200];
    snprintf(msg, sizeof msg,
             "project_noalloc: B*n = %lld pairs exceeds the static scratch limit of %lld pairs; "
             "use splax_project",
             static_cast<long long>(total), static_cast<long long>(kNoAllocMaxPairs));
    return record_error(SPLAX_ERR_INVALID_ARGUMENT, msg);
  }
  const int64_t B = total / n;
  auto rows_ok = [&](int64_t r) { return r == n || r == total; };
  if (!rows_ok(means3d_rows) || !rows_ok(scales_rows) || !rows_ok(quats_rows) ||
      !rows_ok(opacities_rows) || !(viewmat_rows == 4 || viewmat_rows == 4 * B))
    return record_error(SPLAX_ERR_INVALID_ARGUMENT,
                        "project_noalloc: operand rows must be n or B*n (viewmat 4 or 4B)");
  if (has_transforms &&
      (num_transforms <= 0 ||
       !(transforms_rows == num_transforms || transforms_rows == num_transforms * B) ||
       transform_ids == nullptr))
    return record_error(SPLAX_ERR_INVALID_ARGUMENT,
                        "project_noalloc: transforms must have K or B*K matrices");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_error(SPLAX_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return record_error(SPLAX_ERR_INVALID_ARGUMENT, "project_noalloc: device index above 63");
  unsigned long long* words = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      // host code only holds a stand-in for the array: resolve its device address once,
      // on this device
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess)
        return record_error(SPLAX_ERR_CUDA, cudaGetErrorString(e));
      g_noalloc_ptr[dev] = static_cast<unsigned long long*>(p);
    }
    words = g_noalloc_ptr[dev];
  }
  const int64_t tiles = project_scan_tiles(total);
  // the array keeps the previous call's words: clear ticket, error word and this call's tiles
  e = cudaMemsetAsync(words, 0, sizeof(unsigned long long) * (tiles + 2), stream);
  if (e != cudaSuccess) return record_error(SPLAX_ERR_CUDA, cudaGetErrorString(e));
  ProjectArgs a;
  a.means = means3d;
  a.scales = scales;
  a.quats = quats_xyzw;
  a.viewmat = viewmat;
  a.opacities = opacities;
  a.transforms = gaussian_transforms;
  a.transform_ids = transform_ids;
  a.n = n;
  a.total = total;
  a.num_transforms = num_transforms;
  a.has_transforms = has_transforms != 0;
  a.sel_means = means3d_rows > n;
  a.sel_scales = scales_rows > n;
  a.sel_quats = quats_rows > n;
  a.sel_view = viewmat_rows > 4;
  a.sel_opac = opacities_rows > n;
  a.sel_transforms = transforms_rows > num_transforms;
  a.img_h = img_h;
  a.img_w = img_w;
  a.fx = fx;
  a.fy = fy;
  a.cx = cx;
  a.cy = cy;
  a.glob_scale = glob_scale;
  a.clip_thresh = clip_thresh;
  a.xys = xys;
  a.depths = depths;
  a.radii = radii;
  a.conics = conics;
  a.num_tiles_hit = num_tiles_hit;
  a.cum_tiles_hit = cum_tiles_hit;
  launch_project_fwd(a, words + 2, reinterpret_cast<int*>(words),
                     reinterpret_cast<unsigned*>(words + 1), stream);
  e = cudaGetLastError();
  if (e != cudaSuccess) return record_error(SPLAX_ERR_CUDA, cudaGetErrorString(e));
  const char* sync = getenv("SPLAX_SYNC_CHECK");
  if (sync && sync[0] == '1') {
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return record_error(SPLAX_ERR_CUDA, cudaGetErrorString(e));
    unsigned w = 0;
    e = cudaMemcpy(&w, words + 1, sizeof(unsigned), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return record_error(SPLAX_ERR_CUDA, cudaGetErrorString(e));
    if (w & kErrCountOverflow)
      return record_error(SPLAX_ERR_COUNT_OVERFLOW,
                          "project_noalloc: the intersection count exceeds the int32 range");
    if (w) return record_error(SPLAX_ERR_DEVICE, "project_noalloc: a look-back wait gave up");
  }
  return SPLAX_OK;
}
