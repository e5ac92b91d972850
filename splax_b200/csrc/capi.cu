// C ABI of libsplax_b200 (declared in include/splax_b200.h): argument validation, the
// per-device grow-only scratch cache (splax/_cache.py:52-164), the host orchestration of
// sort_and_bin with its single count readback (splax/_rasterize/_sort/_sort.py:29-171) and
// the launch sequences of the six FFI targets.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/splax_b200.h"
#include "common.cuh"
#include "kernels.h"

#include <nvtx3/nvToolsExt.h>

// One NVTX range per C entry point (a no-op unless a profiler is attached), so a timeline shows
// the reference's FFI targets around their kernels.
struct NvtxScope {
  explicit NvtxScope(const char* name) { nvtxRangePushA(name); }
  ~NvtxScope() { nvtxRangePop(); }
};
#define SPLAX_NVTX(name) NvtxScope splax_nvtx_scope_(name)

namespace splax {
namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? SPLAX_ERR_OUT_OF_MEMORY : SPLAX_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

#define SPLAX_CUDA(call)                                  \
  do {                                                    \
    cudaError_t e_ = (call);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);   \
  } while (0)

std::atomic<int64_t> g_fail_after{-1};

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

cudaError_t buf_free(DevBuf& b) {
  cudaError_t e = cudaSuccess;
  if (b.p) e = cudaFree(b.p);
  b.p = nullptr;
  b.bytes = 0;
  return e;
}

// Grow-only device buffer; contents are not preserved across growth.
cudaError_t buf_reserve(DevBuf& b, size_t bytes) {
  if (bytes == 0) bytes = 16;
  if (b.p && b.bytes >= bytes) return cudaSuccess;
  buf_free(b);
  int64_t left = g_fail_after.load();
  if (left == 0) {
    g_fail_after.store(-1);
    return cudaErrorMemoryAllocation;
  }
  if (left > 0) g_fail_after.store(left - 1);
  cudaError_t e = cudaMalloc(&b.p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    b.p = nullptr;
    return e;
  }
  b.bytes = bytes;
  return cudaSuccess;
}

constexpr double kScratchHeadroom = 1.25;  // splax/_cache.py:149

// ------------------------------------------------------------------ profiling (opt-in)
std::atomic<bool> g_timing{false};
std::atomic<uint32_t> g_timing_mask{0xffffffffu};  // bit k: stage kind k is timed
std::atomic<bool> g_count_work{false};
constexpr int kWorkWords = 6;  // device work counters (see DeviceState::work)

enum Kind { kProjectFwd, kProjectBwd, kDepthMinmax, kPairKeys, kPairSort, kPairScan, kEmit,
            kRadixSort, kTileBins, kRasterFwd, kRasterBwd, kLoss, kOptim, kAllReduce,
            kNumKinds };
const char* kKindNames[kNumKinds] = {"project_fwd", "project_bwd", "depth_minmax", "pair_keys",
                                     "pair_sort", "pair_scan", "emit_keys", "radix_sort",
                                     "tile_bins", "raster_fwd", "raster_bwd", "loss", "optim",
                                     "allreduce"};

// CUDA-event timing of each launch sequence on the stream it runs on, resolved lazily.
struct KernelTimer {
  struct Pending {
    int kind;
    int kernels;
    cudaEvent_t a, b;
  };
  std::vector<cudaEvent_t> pool;
  std::vector<Pending> pending;
  double ms[kNumKinds] = {};
  int64_t launches[kNumKinds] = {};
  int64_t kernels[kNumKinds] = {};

  cudaEvent_t get() {
    cudaEvent_t e = nullptr;
    if (!pool.empty()) {
      e = pool.back();
      pool.pop_back();
    } else {
      cudaEventCreate(&e);
    }
    return e;
  }
  bool open = false;  // the last begin() recorded an event that end() must close
  void begin(int kind, int nkernels, cudaStream_t s) {
    open = g_timing.load(std::memory_order_relaxed) &&
           (g_timing_mask.load(std::memory_order_relaxed) >> kind & 1u) != 0;
    if (!open) return;
    Pending p{kind, nkernels, get(), get()};
    cudaEventRecord(p.a, s);
    pending.push_back(p);
  }
  void end(cudaStream_t s) {
    if (!open || pending.empty()) return;
    open = false;
    cudaEventRecord(pending.back().b, s);
  }
  void collect() {
    for (const Pending& p : pending) {
      float t = 0.0f;
      if (cudaEventSynchronize(p.b) == cudaSuccess && cudaEventElapsedTime(&t, p.a, p.b) == cudaSuccess) {
        ms[p.kind] += t;
        launches[p.kind] += 1;
        kernels[p.kind] += p.kernels;
      }
      pool.push_back(p.a);
      pool.push_back(p.b);
    }
    pending.clear();
  }
  void reset() {
    collect();
    for (int k = 0; k < kNumKinds; ++k) {
      ms[k] = 0.0;
      launches[k] = 0;
      kernels[k] = 0;
    }
  }
};

// Host-side work units for the roofline (what the launches processed).
struct WorkUnits {
  int64_t pairs_fwd = 0;       // (camera, gaussian) pairs projected
  int64_t pairs_bwd = 0;       // pairs through the projection backward
  int64_t intersections = 0;   // keys emitted and sorted
  int64_t key_bytes = 0;       // sum of intersections * key size
  int64_t sort_passes = 0;     // sum of intersections * radix passes
  int64_t visible = 0;         // not tracked on the host (device counters below)
  int64_t pixels_fwd = 0, pixels_bwd = 0;
  int64_t bins = 0;
  int64_t sort_reuses = 0;   // backward passes that reused the forward's sort
  int64_t pairs_sorted = 0;  // (camera, gaussian) pairs through the depth-order sort
  int64_t pair_key_bytes = 0;
  int64_t pair_pass_keys = 0;
};

struct SortOut {
  const int32_t* gids = nullptr;
  const uint32_t* keys = nullptr;  // sorted (image | tile) bin keys
  const int32_t* bins = nullptr;
  const float4* records = nullptr;
  int64_t count = 0;
  int32_t tbx = 0, tby = 0, num_tiles = 0;
  int key_bits = 0;  // the reference's key width for this call (32 packed, 64 wide)
  int32_t tile_n_bits = 0, depth_bits = 0;
  const int32_t* depth_mm = nullptr;
};

struct SortIn {
  const float* xys;
  const float* depths;
  const int32_t* radii;
  const float* conics;
  const float* map_opacities;
  int64_t map_rows;
  const float* opacities;
  int64_t opac_rows;
  const float* colors;
  int64_t color_rows;
  const int32_t* cum;
  int64_t n, B;
  int32_t img_h, img_w;
  int key_req;
};

struct DeviceState {
  std::mutex mu;
  int device = -1;
  // scratch entry keyed on the workload signature (B, n, tiles)
  int64_t sig_B = -1, sig_n = -1, sig_T = -1;
  int key_bits = 0;
  int64_t isect_cap = 0;
  DevBuf keys[2], vals[2], records, tile_bins, depth_mm, status;
  DevBuf pkeys[2], pvals[2], poffs, scan_status;  // depth-order sort of the B*n pairs
  DevBuf walk, counts;                             // per-pair walk records and tile counts
  // signature-independent pieces
  DevBuf misc;  // [0] error word, [2..9] sort tile counters, [10] depth span, [11] scan ticket
  DevBuf hist;        // radix histograms and offsets
  DevBuf proj_status; // projection scan look-back words
  int32_t* pinned = nullptr;  // [0] count, [1] error word
  cudaEvent_t ev = nullptr;
  // device work counters: fwd evals, fwd contribs, bwd evals, bwd contribs, bwd warp steps,
  // bwd warp steps with a contribution
  DevBuf work;
  DevBuf loss;  // fused loss: per-CTA fp64 partials, then the completion counter
  DevBuf ssim_partials;  // fused L1 + D-SSIM loss: per-CTA fp64 partial sums
  // .ply loading: two pinned host chunks, two device staging chunks, copy-done events
  void* ply_host[2] = {nullptr, nullptr};
  DevBuf ply_dev[2];
  size_t ply_chunk = 0;
  cudaEvent_t ply_ev[2] = {nullptr, nullptr};
  bool ssim_window = false;  // the SSIM window weights are in this device's constant bank
  KernelTimer timer;
  WorkUnits units;
  // the most recent sort_and_bin result, reusable by a backward over the same inputs
  uint64_t sort_gen = 0;
  bool last_valid = false;
  uint64_t last_gen = 0;
  SortIn last_in{};
  SortOut last_out{};

  unsigned long long* work_fwd() {
    return g_count_work.load() ? static_cast<unsigned long long*>(work.p) : nullptr;
  }
  unsigned long long* work_bwd() {
    return g_count_work.load() ? static_cast<unsigned long long*>(work.p) + 2 : nullptr;
  }

  unsigned* err_word() { return static_cast<unsigned*>(misc.p); }
  int* sort_counters() { return static_cast<int*>(misc.p) + 2; }
  unsigned* span_word() { return static_cast<unsigned*>(misc.p) + 10; }
  int* scan_ticket() { return static_cast<int*>(misc.p) + 11; }
  int32_t* vis_word() { return static_cast<int32_t*>(misc.p) + 12; }  // pairs that hit a tile

  size_t bytes_held() const {
    size_t s = 0;
    for (const DevBuf* b : {&keys[0], &keys[1], &vals[0], &vals[1], &records, &tile_bins,
                            &depth_mm, &status, &pkeys[0], &pkeys[1], &pvals[0], &pvals[1],
                            &poffs, &scan_status, &walk, &counts, &misc, &hist,
                            &proj_status, &loss, &ssim_partials})
      s += b->bytes;
    return s;
  }

  void drop_entry() {
    last_valid = false;
    ++sort_gen;
    for (DevBuf* b : {&keys[0], &keys[1], &vals[0], &vals[1], &records, &tile_bins, &depth_mm,
                      &status, &pkeys[0], &pkeys[1], &pvals[0], &pvals[1], &poffs, &scan_status,
                      &walk, &counts})
      buf_free(*b);
    sig_B = sig_n = sig_T = -1;
    key_bits = 0;
    isect_cap = 0;
  }

  int init() {
    if (ev) return SPLAX_OK;
    SPLAX_CUDA(buf_reserve(misc, 64));
    SPLAX_CUDA(cudaMemset(misc.p, 0, 64));
    SPLAX_CUDA(buf_reserve(hist, sizeof(uint32_t) * 2 * 8 * 256));
    SPLAX_CUDA(buf_reserve(work, kWorkWords * sizeof(unsigned long long)));
    SPLAX_CUDA(cudaMemset(work.p, 0, kWorkWords * sizeof(unsigned long long)));
    SPLAX_CUDA(cudaMallocHost(&pinned, 4 * sizeof(int32_t)));
    SPLAX_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    return SPLAX_OK;
  }
};

std::mutex g_states_mu;
std::vector<std::unique_ptr<DeviceState>> g_states;

int current_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_states_mu);
  if (static_cast<int>(g_states.size()) <= dev) g_states.resize(dev + 1);
  if (!g_states[dev]) {
    g_states[dev] = std::make_unique<DeviceState>();
    g_states[dev]->device = dev;
  }
  *out = g_states[dev].get();
  return SPLAX_OK;
}

int bit_length(int64_t v) {
  int b = 0;
  while (v > 0) {
    ++b;
    v >>= 1;
  }
  return b;
}

const char* describe_device_error(unsigned w) {
  if (w & kErrLookbackTimeout) return "a look-back wait exceeded its iteration limit";
  if (w & kErrEmitCount)
    return "emitted intersections disagree with cum_tiles_hit (geometry, map_opacities and "
           "cum_tiles_hit must come from the same projection)";
  if (w & kErrNegativeDepthKey)
    return "a visible gaussian has a negative depth, which the 64-bit sort key cannot order "
           "(use clip_thresh >= 0)";
  if (w & kErrCountOverflow) return "the intersection count exceeds the int32 range";
  if (w & kErrBinRange) return "a sorted key decoded to a tile bin outside the batch";
  return "unknown device error";
}

int report_device_error(DeviceState& st, unsigned w, cudaStream_t stream) {
  cudaMemsetAsync(st.err_word(), 0, sizeof(unsigned), stream);
  int code = (w & kErrCountOverflow) ? SPLAX_ERR_COUNT_OVERFLOW : SPLAX_ERR_DEVICE;
  return fail(code, std::string("device check failed: ") + describe_device_error(w));
}

// sort_and_bin (splax/_rasterize/_sort/_sort.py:29-171) plus the record packing. The sorted
// order equals the reference's stable sort of (image | tile | depth key) keys, produced as a
// stable depth-order sort of the B*n pairs followed by a stable sort of the intersections by
// their (image | tile) field alone.
int sort_and_bin(DeviceState& st, const SortIn& in, cudaStream_t stream, SortOut& out) {
  int rc = st.init();
  if (rc) return rc;
  st.last_valid = false;  // the scratch is about to be rewritten
  ++st.sort_gen;
  const int32_t tbx = (in.img_w + kBlockWidth - 1) / kBlockWidth;
  const int32_t tby = (in.img_h + kBlockWidth - 1) / kBlockWidth;
  const int64_t num_tiles = static_cast<int64_t>(tbx) * tby;
  const int tile_n_bits = bit_length(num_tiles - 1);
  const int image_n_bits = bit_length(in.B - 1);
  const int upper = tile_n_bits + image_n_bits;
  const int depth_bits = 31 - upper;
  const bool packed = in.key_req == 0 ? depth_bits >= 16 : in.key_req == 32;
  if (!packed && upper > 32) {
    char msg[256];
    snprintf(msg, sizeof msg,
             "batched intersection key overflow: image_n_bits(%d) + tile_n_bits(%d) = %d > 32 "
             "(batch B=%lld, n_tiles=%lld). Reduce batch size or resolution.",
             image_n_bits, tile_n_bits, upper, static_cast<long long>(in.B),
             static_cast<long long>(num_tiles));
    return fail(SPLAX_ERR_KEY_OVERFLOW, msg);
  }
  if (packed && depth_bits < 1)
    return fail(SPLAX_ERR_KEY_OVERFLOW, "32-bit keys requested but image and tile ids leave no "
                                        "depth bits");
  const int64_t total = in.B * in.n;
  const int64_t bins_len = in.B * num_tiles;
  // scratch entry for this signature
  if (st.sig_B != in.B || st.sig_n != in.n || st.sig_T != num_tiles) {
    SPLAX_CUDA(cudaStreamSynchronize(stream));
    st.drop_entry();
    cudaError_t e;
    const int64_t ptiles = sorted_offsets_tiles(total);
    if ((e = buf_reserve(st.tile_bins, sizeof(int2) * bins_len)) != cudaSuccess ||
        (e = buf_reserve(st.depth_mm, sizeof(int32_t) * 2 * in.B)) != cudaSuccess ||
        (e = buf_reserve(st.records, sizeof(float4) * kRecordFloat4 * total)) != cudaSuccess ||
        (e = buf_reserve(st.pkeys[0], sizeof(uint64_t) * total)) != cudaSuccess ||
        (e = buf_reserve(st.pkeys[1], sizeof(uint64_t) * total)) != cudaSuccess ||
        (e = buf_reserve(st.pvals[0], sizeof(int32_t) * total)) != cudaSuccess ||
        (e = buf_reserve(st.pvals[1], sizeof(int32_t) * total)) != cudaSuccess ||
        (e = buf_reserve(st.poffs, sizeof(int32_t) * total)) != cudaSuccess ||
        (e = buf_reserve(st.scan_status, sizeof(unsigned long long) * ptiles)) != cudaSuccess ||
        (e = buf_reserve(st.walk, 2 * sizeof(float4) * total)) != cudaSuccess ||
        (e = buf_reserve(st.counts, sizeof(int32_t) * total)) != cudaSuccess) {
      st.drop_entry();
      return cuda_fail(e, "scratch allocation (tile bins, depth ranges, records, pair order)");
    }
    st.sig_B = in.B;
    st.sig_n = in.n;
    st.sig_T = num_tiles;
  }
  // count-independent work first, then the one device-to-host sync: intersection count,
  // device error word and (wide keys) the largest per-image depth-bit span
  int32_t* depth_mm = static_cast<int32_t*>(st.depth_mm.p);
  st.timer.begin(kDepthMinmax, packed ? 2 : 3, stream);
  launch_depth_minmax(in.depths, in.radii, total, in.n, static_cast<int32_t>(in.B), depth_mm,
                      stream);
  if (!packed) launch_depth_span(depth_mm, static_cast<int32_t>(in.B), st.span_word(), stream);
  st.timer.end(stream);
  SPLAX_CUDA(cudaMemcpyAsync(&st.pinned[0], in.cum + (total - 1), sizeof(int32_t),
                             cudaMemcpyDeviceToHost, stream));
  SPLAX_CUDA(cudaMemcpyAsync(&st.pinned[1], st.err_word(), sizeof(int32_t),
                             cudaMemcpyDeviceToHost, stream));
  SPLAX_CUDA(cudaMemcpyAsync(&st.pinned[2], st.span_word(), sizeof(int32_t),
                             cudaMemcpyDeviceToHost, stream));
  SPLAX_CUDA(cudaEventRecord(st.ev, stream));
  {
    const ClearSpan span = {st.tile_bins.p, sizeof(int2) * static_cast<size_t>(bins_len)};
    launch_clear(&span, 1, stream);
  }

  SortScratch ss;
  ss.hist = static_cast<uint32_t*>(st.hist.p);
  ss.tile_counters = st.sort_counters();
  ss.err = st.err_word();
  int32_t* offsets = static_cast<int32_t*>(st.poffs.p);
  const int32_t* perm = nullptr;
  int pair_bits = 0;
  bool pair64 = false;
  // 1. pairs in (image, depth key) order. Nothing here depends on the intersection count, so
  // with packed keys (the key layout known on the host) this stage is queued before the host
  // waits for the count and keeps the GPU busy across that wait.
  auto pair_stage = [&](int key_shift) -> int {
    pair_bits = image_n_bits + key_shift;
    // 64-bit pair keys from 32 significant bits: the all-ones key marks pairs left out
    pair64 = pair_bits > 31;
    const int64_t t_pairs = (total + sort_tile_items(pair64) - 1) / sort_tile_items(pair64);
    // two halves: consecutive passes alternate between them (radix_sort_pairs)
    const size_t need = 2 * sizeof(unsigned long long) * kRadixMaxDigits * t_pairs;
    if (st.status.bytes < need) {
      SPLAX_CUDA(cudaStreamSynchronize(stream));
      cudaError_t e = buf_reserve(st.status, need);
      if (e != cudaSuccess) {
        st.drop_entry();
        return cuda_fail(e, "sort look-back allocation");
      }
    }
    ss.status = static_cast<unsigned long long*>(st.status.p);
    ss.status_words = static_cast<int64_t>(st.status.bytes / sizeof(unsigned long long));
    PairKeyArgs pa;
    pa.depths = in.depths;
    pa.radii = in.radii;
    pa.depth_mm = depth_mm;
    pa.n = in.n;
    pa.total = total;
    pa.packed = packed;
    pa.depth_bits = depth_bits;
    pa.key_shift = key_shift;
    pa.err = st.err_word();
    pa.xys = in.xys;
    pa.conics = in.conics;
    pa.cum = in.cum;
    pa.map_opacities = in.map_opacities;
    pa.map_opac_rows = in.map_rows;
    pa.opacities = in.opacities;
    pa.opac_rows = in.opac_rows;
    pa.colors = in.colors;
    pa.color_rows = in.color_rows;
    pa.counts = static_cast<int32_t*>(st.counts.p);
    pa.walk = static_cast<float4*>(st.walk.p);
    pa.records = in.colors ? static_cast<float4*>(st.records.p) : nullptr;
    st.timer.begin(kPairKeys, 1, stream);
    launch_pair_keys(pa, pair64, st.pkeys[0].p, static_cast<int32_t*>(st.pvals[0].p), stream);
    st.timer.end(stream);
    ss.keys[0] = st.pkeys[0].p;
    ss.keys[1] = st.pkeys[1].p;
    ss.vals[0] = static_cast<int32_t*>(st.pvals[0].p);
    ss.vals[1] = static_cast<int32_t*>(st.pvals[1].p);
    const int pair_passes = radix_passes(pair_bits);
    st.timer.begin(kPairSort, total > 1 && pair_passes ? 2 + pair_passes : 0, stream);
    // only the V pairs that hit a tile are sorted; V stays on the device
    ss.filter_sentinel = true;
    ss.vcount = st.vis_word();
    const int pfin = radix_sort_pairs(ss, pair64, total, pair_bits, stream);
    ss.filter_sentinel = false;
    ss.vcount = nullptr;
    st.timer.end(stream);
    perm = ss.vals[pfin];
    st.timer.begin(kPairScan, 1, stream);
    launch_sorted_offsets(perm, static_cast<const int32_t*>(st.counts.p), total, st.vis_word(),
                          offsets, static_cast<unsigned long long*>(st.scan_status.p),
                          st.scan_ticket(), st.err_word(), stream);
    st.timer.end(stream);
    return SPLAX_OK;
  };
  if (packed) {
    rc = pair_stage(depth_bits);
    if (rc) return rc;
  }
  SPLAX_CUDA(cudaEventSynchronize(st.ev));
  const unsigned werr = static_cast<unsigned>(st.pinned[1]);
  if (werr) return report_device_error(st, werr, stream);
  const int64_t count = static_cast<int64_t>(st.pinned[0]);
  if (count < 0)
    return fail(SPLAX_ERR_COUNT_OVERFLOW,
                "cum_tiles_hit[-1] is negative: the intersection count overflowed int32");
  const int kb = packed ? 32 : 64;
  const int bin_bits = upper;
  if (st.isect_cap < count) {
    const int64_t cap = std::max<int64_t>(static_cast<int64_t>(count * kScratchHeadroom) + 1,
                                          st.isect_cap);
    SPLAX_CUDA(cudaStreamSynchronize(stream));
    for (DevBuf* b : {&st.keys[0], &st.keys[1], &st.vals[0], &st.vals[1]}) buf_free(*b);
    st.isect_cap = 0;
    cudaError_t e;
    if ((e = buf_reserve(st.keys[0], sizeof(uint32_t) * cap)) != cudaSuccess ||
        (e = buf_reserve(st.keys[1], sizeof(uint32_t) * cap)) != cudaSuccess ||
        (e = buf_reserve(st.vals[0], sizeof(int32_t) * cap)) != cudaSuccess ||
        (e = buf_reserve(st.vals[1], sizeof(int32_t) * cap)) != cudaSuccess) {
      st.drop_entry();
      return cuda_fail(e, "sort scratch allocation");
    }
    st.isect_cap = cap;
  }
  st.key_bits = kb;
  out.tbx = tbx;
  out.tby = tby;
  out.num_tiles = static_cast<int32_t>(num_tiles);
  out.key_bits = kb;
  out.tile_n_bits = tile_n_bits;
  out.depth_bits = depth_bits;
  out.depth_mm = depth_mm;
  out.count = count;
  out.bins = static_cast<const int32_t*>(st.tile_bins.p);
  out.records = static_cast<const float4*>(st.records.p);
  out.gids = static_cast<const int32_t*>(st.vals[0].p);
  out.keys = static_cast<const uint32_t*>(st.keys[0].p);
  if (count == 0) {
    st.last_valid = true;
    st.last_gen = st.sort_gen;
    st.last_in = in;
    st.last_out = out;
    return SPLAX_OK;
  }
  if (!packed) {
    // wide keys: the pair key's depth field is as wide as the largest per-image span
    rc = pair_stage(bit_length(static_cast<uint32_t>(st.pinned[2])));
    if (rc) return rc;
  }
  {
    // look-back words of the intersection sort
    const int64_t t_bins = (st.isect_cap + sort_tile_items(false) - 1) / sort_tile_items(false);
    const size_t need = 2 * sizeof(unsigned long long) * kRadixMaxDigits * t_bins;
    if (st.status.bytes < need) {
      SPLAX_CUDA(cudaStreamSynchronize(stream));
      cudaError_t e = buf_reserve(st.status, need);
      if (e != cudaSuccess) {
        st.drop_entry();
        return cuda_fail(e, "sort look-back allocation");
      }
      ss.status = static_cast<unsigned long long*>(st.status.p);
      ss.status_words = static_cast<int64_t>(st.status.bytes / sizeof(unsigned long long));
    }
  }

  // 2. emission in pair order: (image | tile) keys, flat ids, blend records
  EmitArgs ea;
  ea.perm = perm;
  ea.offsets = offsets;
  ea.counts = static_cast<const int32_t*>(st.counts.p);
  ea.walk = static_cast<const float4*>(st.walk.p);
  ea.total = total;
  ea.dtotal = st.vis_word();
  ea.count = count;
  ea.tile_n_bits = tile_n_bits;
  ea.tbx = tbx;
  ea.tby = tby;
  ea.keys = static_cast<uint32_t*>(st.keys[0].p);
  ea.vals = static_cast<int32_t*>(st.vals[0].p);
  ea.err = st.err_word();
  st.timer.begin(kEmit, 1, stream);
  launch_emit(ea, stream);
  st.timer.end(stream);

  // 3. stable sort of the intersections by (image | tile)
  ss.keys[0] = st.keys[0].p;
  ss.keys[1] = st.keys[1].p;
  ss.vals[0] = static_cast<int32_t*>(st.vals[0].p);
  ss.vals[1] = static_cast<int32_t*>(st.vals[1].p);
  const int passes = radix_passes(bin_bits);
  st.timer.begin(kRadixSort, count > 1 && passes ? 2 + passes : 0, stream);
  const int fin = radix_sort_pairs(ss, false, count, bin_bits, stream);
  st.timer.end(stream);
  out.gids = ss.vals[fin];
  out.keys = static_cast<const uint32_t*>(ss.keys[fin]);
  st.timer.begin(kTileBins, 1, stream);
  launch_tile_bins(out.keys, count, tile_n_bits, static_cast<int32_t>(num_tiles), bins_len,
                   static_cast<int32_t*>(st.tile_bins.p), st.err_word(), stream);
  st.timer.end(stream);
  SPLAX_CUDA(cudaGetLastError());
  st.units.intersections += count;
  st.units.key_bytes += count * static_cast<int64_t>(sizeof(uint32_t));
  st.units.sort_passes += count > 1 ? count * passes : 0;
  st.units.bins += bins_len;
  // pairs that entered the depth sort: read back only in the instrumented (work-count) mode
  int64_t sorted_pairs = total;
  if (g_count_work.load()) {
    int32_t v = 0;
    SPLAX_CUDA(cudaMemcpyAsync(&v, st.vis_word(), sizeof(int32_t), cudaMemcpyDeviceToHost,
                               stream));
    SPLAX_CUDA(cudaStreamSynchronize(stream));
    sorted_pairs = v;
  }
  st.units.pairs_sorted += sorted_pairs;
  st.units.pair_key_bytes += sorted_pairs * (pair64 ? 8 : 4);
  st.units.pair_pass_keys += sorted_pairs > 1 ? sorted_pairs * radix_passes(pair_bits) : 0;
  st.last_valid = true;
  st.last_gen = st.sort_gen;
  st.last_in = in;
  st.last_out = out;
  return SPLAX_OK;
}

// Sort reuse between a forward and its backward: the forward leaves its sort's token in the
// calling thread; the caller re-arms it before the backward, which then skips sort_and_bin when
// the token is still the device's latest sort and every input pointer and size is identical.
thread_local int64_t g_last_sort_token = -1;
thread_local int64_t g_armed_sort_token = -1;

bool same_sort_inputs(const SortIn& a, const SortIn& b) {
  return a.xys == b.xys && a.depths == b.depths && a.radii == b.radii && a.conics == b.conics &&
         a.map_opacities == b.map_opacities && a.map_rows == b.map_rows &&
         a.opacities == b.opacities && a.opac_rows == b.opac_rows && a.colors == b.colors &&
         a.color_rows == b.color_rows && a.cum == b.cum && a.n == b.n && a.B == b.B &&
         a.img_h == b.img_h && a.img_w == b.img_w && a.key_req == b.key_req;
}

bool sync_check_enabled() {
  static const bool on = [] {
    const char* v = getenv("SPLAX_SYNC_CHECK");
    return v && v[0] == '1';
  }();
  return on;
}

int finish(DeviceState& st, cudaStream_t stream) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  if (!sync_check_enabled()) return SPLAX_OK;
  SPLAX_CUDA(cudaStreamSynchronize(stream));
  unsigned w = 0;
  SPLAX_CUDA(cudaMemcpy(&w, st.err_word(), sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (w) return report_device_error(st, w, stream);
  return SPLAX_OK;
}

bool bad_rows(int64_t rows, int64_t n, int64_t total) {
  // a per-gaussian operand is shared (n rows) or batched (total rows)
  return !(rows == n || rows == total);
}

int rasterize_common(const float* colors, int64_t colors_rows, const float* opacities,
                     int64_t opacities_rows, const float* map_opacities, int64_t map_rows,
                     const float* background, int64_t background_rows, const float* xys,
                     const float* depths, const int32_t* radii, const float* conics,
                     const int32_t* cum, int64_t geom_rows, int32_t n, int32_t img_h,
                     int32_t img_w, int64_t out_rows, int32_t key_bits, float* final_Ts,
                     int32_t* final_idx, float* out_img, float* out_depth, cudaStream_t stream) {
  if (n <= 0 || img_h <= 0 || img_w <= 0 || out_rows <= 0 || out_rows % img_h != 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize: invalid n, image size or output rows");
  const int64_t B = out_rows / img_h;
  if (geom_rows != B * n)
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "rasterize: projected geometry must have B*n rows for B = out_rows / img_h");
  if (bad_rows(colors_rows, n, geom_rows) || bad_rows(opacities_rows, n, geom_rows) ||
      bad_rows(map_rows, n, geom_rows) || !(background_rows == 1 || background_rows == B))
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "rasterize: operand rows must be n or B*n (background 1 or B)");
  if (key_bits != 0 && key_bits != 32 && key_bits != 64)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize: key_bits must be 0, 32 or 64");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  SortIn in{xys, depths, radii, conics, map_opacities, map_rows, opacities, opacities_rows,
            colors, colors_rows, cum, n, B, img_h, img_w, key_bits};
  SortOut so;
  g_last_sort_token = -1;
  rc = sort_and_bin(*st, in, stream, so);
  if (rc) return rc;
  g_last_sort_token = static_cast<int64_t>(st->sort_gen);
  RasterFwdArgs ra;
  ra.img_h = img_h;
  ra.img_w = img_w;
  ra.tbx = so.tbx;
  ra.num_tiles = so.num_tiles;
  ra.num_images = B;
  ra.tile_bins = so.bins;
  ra.gids = so.gids;
  ra.records = so.records;
  ra.num_records = B * static_cast<int64_t>(n);
  ra.background = background;
  ra.sel_bg = background_rows > 1;
  ra.final_Ts = final_Ts;
  ra.final_idx = final_idx;
  ra.out_img = out_img;
  ra.out_depth = out_depth;
  ra.work = st->work_fwd();
  st->timer.begin(kRasterFwd, 1, stream);
  launch_raster_fwd(ra, stream);
  st->timer.end(stream);
  st->units.pixels_fwd += B * static_cast<int64_t>(img_h) * img_w;
  return finish(*st, stream);
}

int rasterize_bwd_common(const float* colors, int64_t colors_rows, const float* opacities,
                         int64_t opacities_rows, const float* map_opacities, int64_t map_rows,
                         const float* background, int64_t background_rows, const float* xys,
                         const float* depths, const int32_t* radii, const float* conics,
                         const int32_t* cum, int64_t geom_rows, const float* final_Ts,
                         const int32_t* final_idx, const float* v_out_img, int64_t v_out_rows,
                         const float* v_out_depth, int64_t v_out_depth_rows, int32_t n,
                         int32_t img_h, int32_t img_w, int64_t grad_rows, int32_t key_bits,
                         float* v_colors, float* v_opacity, float* v_xy, float* v_conic,
                         float* v_depths, bool fold_colors, bool fold_opacity,
                         cudaStream_t stream) {
  if (n <= 0 || img_h <= 0 || img_w <= 0 || geom_rows <= 0 || geom_rows % n != 0 ||
      grad_rows <= 0 || grad_rows % n != 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize_bwd: invalid n, image size or rows");
  const int64_t B_geom = geom_rows / n, B_out = grad_rows / n;
  if (B_geom != 1 && B_geom != B_out)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize_bwd: geometry batch must be 1 or B_out");
  if (v_out_rows <= 0 || v_out_rows % img_h != 0 ||
      (v_out_depth && (v_out_depth_rows <= 0 || v_out_depth_rows % img_h != 0)))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize_bwd: cotangent rows must be k*img_h");
  if (bad_rows(colors_rows, n, geom_rows) || bad_rows(opacities_rows, n, geom_rows) ||
      bad_rows(map_rows, n, geom_rows) || !(background_rows == 1 || background_rows == B_out))
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "rasterize_bwd: operand rows must be n or B*n (background 1 or B_out)");
  if (key_bits != 0 && key_bits != 32 && key_bits != 64)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize_bwd: key_bits must be 0, 32 or 64");
  if ((fold_colors && colors_rows != n) || (fold_opacity && opacities_rows != n))
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "rasterize_bwd: folded colour / opacity gradients need shared operands");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  {
    const ClearSpan spans[5] = {
        {v_colors, sizeof(float) * 3 * static_cast<size_t>(fold_colors ? n : grad_rows)},
        {v_opacity, sizeof(float) * static_cast<size_t>(fold_opacity ? n : grad_rows)},
        {v_xy, sizeof(float) * 2 * static_cast<size_t>(grad_rows)},
        {v_conic, sizeof(float) * 3 * static_cast<size_t>(grad_rows)},
        {v_depths, v_depths ? sizeof(float) * static_cast<size_t>(grad_rows) : 0}};
    launch_clear(spans, 5, stream);
  }
  SortIn in{xys, depths, radii, conics, map_opacities, map_rows, opacities, opacities_rows,
            colors, colors_rows, cum, n, B_geom, img_h, img_w, key_bits};
  SortOut so;
  const int64_t armed = g_armed_sort_token;
  g_armed_sort_token = -1;
  if (armed >= 0 && st->last_valid && static_cast<uint64_t>(armed) == st->last_gen &&
      same_sort_inputs(st->last_in, in)) {
    so = st->last_out;
    st->units.sort_reuses += 1;
  } else {
    rc = sort_and_bin(*st, in, stream, so);
    if (rc) return rc;
  }
  if (so.count == 0) return finish(*st, stream);
  RasterBwdArgs ba;
  ba.img_h = img_h;
  ba.img_w = img_w;
  ba.tbx = so.tbx;
  ba.num_tiles = so.num_tiles;
  ba.n = n;
  ba.B_out = B_out;
  ba.sel_geom = B_geom > 1;
  ba.sel_bg = background_rows > 1;
  ba.vout_rows = v_out_rows;
  ba.vdepth_rows = v_out_depth_rows;
  ba.tile_bins = so.bins;
  ba.gids = so.gids;
  ba.records = so.records;
  ba.num_records = B_geom * static_cast<int64_t>(n);
  ba.background = background;
  ba.final_Ts = final_Ts;
  ba.final_idx = final_idx;
  ba.v_out_img = v_out_img;
  ba.v_out_depth = v_out_depth;
  ba.v_colors = v_colors;
  ba.v_opacity = v_opacity;
  ba.v_xy = v_xy;
  ba.v_conic = v_conic;
  ba.v_depths = v_depths;
  ba.fold_colors = fold_colors;
  ba.fold_opacity = fold_opacity;
  ba.work = st->work_bwd();
  st->timer.begin(kRasterBwd, 1, stream);
  launch_raster_bwd(ba, stream);
  st->timer.end(stream);
  st->units.pixels_bwd += B_out * static_cast<int64_t>(img_h) * img_w;
  return finish(*st, stream);
}

}  // namespace

int record_error(int code, const char* msg) { return fail(code, msg); }

}  // namespace splax

using namespace splax;

extern "C" {

const char* splax_last_error(void) { return g_last_error.c_str(); }

const char* splax_version(void) { return "splax_b200 0.1.0 (sm_100a)"; }

static int project_impl(const float* means3d, int64_t means3d_rows, const float* scales,
                        int64_t scales_rows, const float* quats_xyzw, int64_t quats_rows,
                        const float* viewmat, int64_t viewmat_rows, const float* opacities,
                        int64_t opacities_rows, const float* gaussian_transforms,
                        int64_t transforms_rows, const int32_t* transform_ids,
                        int32_t num_gaussians, int32_t num_transforms, int32_t has_transforms,
                        int32_t img_h, int32_t img_w, float fx, float fy, float cx, float cy,
                        float glob_scale, float clip_thresh, int64_t total, float* xys,
                        float* depths, int32_t* radii, float* conics, int32_t* num_tiles_hit,
                        int32_t* cum_tiles_hit, int32_t quats_wxyz, float aa_eps,
                        float aa_eps2, float* rho, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t n = num_gaussians;
  if (n <= 0 || total <= 0 || total % n != 0 || img_h <= 0 || img_w <= 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "project: invalid num_gaussians, total or image size");
  const int64_t B = total / n;
  if (bad_rows(means3d_rows, n, total) || bad_rows(scales_rows, n, total) ||
      bad_rows(quats_rows, n, total) || bad_rows(opacities_rows, n, total) ||
      !(viewmat_rows == 4 || viewmat_rows == 4 * B))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "project: operand rows must be n or B*n (viewmat 4 or 4B)");
  if (has_transforms &&
      (num_transforms <= 0 ||
       !(transforms_rows == num_transforms || transforms_rows == num_transforms * B) ||
       transform_ids == nullptr))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "project: transforms must have K or B*K matrices");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  const int64_t tiles = project_scan_tiles(total);
  // [ticket (8 bytes)] [look-back words]
  SPLAX_CUDA(buf_reserve(st->proj_status, sizeof(unsigned long long) * (tiles + 1)));
  {
    const ClearSpan span = {st->proj_status.p, sizeof(unsigned long long) * (tiles + 1)};
    launch_clear(&span, 1, stream);
  }
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
  a.rho = rho;
  a.aa_eps = aa_eps;
  a.aa_eps2 = aa_eps2;
  a.quats_wxyz = quats_wxyz != 0;
  unsigned long long* words = static_cast<unsigned long long*>(st->proj_status.p);
  st->timer.begin(kProjectFwd, 1, stream);
  launch_project_fwd(a, words + 1, reinterpret_cast<int*>(words), st->err_word(), stream);
  st->timer.end(stream);
  st->units.pairs_fwd += total;
  return finish(*st, stream);
}

int splax_project(const float* means3d, int64_t means3d_rows, const float* scales,
                  int64_t scales_rows, const float* quats_xyzw, int64_t quats_rows,
                  const float* viewmat, int64_t viewmat_rows, const float* opacities,
                  int64_t opacities_rows, const float* gaussian_transforms,
                  int64_t transforms_rows, const int32_t* transform_ids, int32_t num_gaussians,
                  int32_t num_transforms, int32_t has_transforms, int32_t img_h, int32_t img_w,
                  float fx, float fy, float cx, float cy, float glob_scale, float clip_thresh,
                  int64_t total, float* xys, float* depths, int32_t* radii, float* conics,
                  int32_t* num_tiles_hit, int32_t* cum_tiles_hit, void* stream) {
  SPLAX_NVTX("splax_project");
  return project_impl(means3d, means3d_rows, scales, scales_rows, quats_xyzw, quats_rows,
                      viewmat, viewmat_rows, opacities, opacities_rows, gaussian_transforms,
                      transforms_rows, transform_ids, num_gaussians, num_transforms,
                      has_transforms, img_h, img_w, fx, fy, cx, cy, glob_scale, clip_thresh,
                      total, xys, depths, radii, conics, num_tiles_hit, cum_tiles_hit, 0, 0.0f,
                      0.0f, nullptr, stream);
}

int splax_project_ex(const float* means3d, int64_t means3d_rows, const float* scales,
                     int64_t scales_rows, const float* quats, int64_t quats_rows,
                     const float* viewmat, int64_t viewmat_rows, const float* opacities,
                     int64_t opacities_rows, const float* gaussian_transforms,
                     int64_t transforms_rows, const int32_t* transform_ids,
                     int32_t num_gaussians, int32_t num_transforms, int32_t has_transforms,
                     int32_t img_h, int32_t img_w, float fx, float fy, float cx, float cy,
                     float glob_scale, float clip_thresh, int64_t total, float* xys,
                     float* depths, int32_t* radii, float* conics, int32_t* num_tiles_hit,
                     int32_t* cum_tiles_hit, int32_t quats_wxyz, float aa_eps, float aa_eps2,
                     float* rho, void* stream) {
  SPLAX_NVTX("splax_project_ex");
  return project_impl(means3d, means3d_rows, scales, scales_rows, quats, quats_rows, viewmat,
                      viewmat_rows, opacities, opacities_rows, gaussian_transforms,
                      transforms_rows, transform_ids, num_gaussians, num_transforms,
                      has_transforms, img_h, img_w, fx, fy, cx, cy, glob_scale, clip_thresh,
                      total, xys, depths, radii, conics, num_tiles_hit, cum_tiles_hit,
                      quats_wxyz, aa_eps, aa_eps2, rho, stream);
}
static int project_bwd_impl(const float* means3d, int64_t means3d_rows, const float* scales,
                            int64_t scales_rows, const float* quats_xyzw, int64_t quats_rows,
                            const float* viewmat, int64_t viewmat_rows, const int32_t* radii,
                            int64_t radii_rows, const float* conics, int64_t conics_rows,
                            const float* v_xy, int64_t v_xy_rows, const float* v_depth,
                            int64_t v_depth_rows, const float* v_conic, int64_t v_conic_rows,
                            const float* v_rho, int64_t v_rho_rows, float aa_eps, float aa_eps2,
                            const float* gaussian_transforms, int64_t transforms_rows,
                            const int32_t* transform_ids, int32_t num_gaussians,
                            int32_t num_transforms, int32_t has_transforms, float fx, float fy,
                            float glob_scale, int64_t out_rows, int32_t quats_wxyz,
                            int32_t fold_batch, float* v_mean3d, float* v_scale, float* v_quat,
                            float* v_viewmat, float* v_transforms, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t n = num_gaussians;
  if (n <= 0 || out_rows <= 0 || out_rows % n != 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "project_bwd: invalid num_gaussians or output rows");
  const int64_t B = out_rows / n;
  if (bad_rows(means3d_rows, n, out_rows) || bad_rows(scales_rows, n, out_rows) ||
      bad_rows(quats_rows, n, out_rows) || bad_rows(radii_rows, n, out_rows) ||
      bad_rows(conics_rows, n, out_rows) || (v_xy && bad_rows(v_xy_rows, n, out_rows)) ||
      (v_depth && bad_rows(v_depth_rows, n, out_rows)) || bad_rows(v_conic_rows, n, out_rows) ||
      (v_rho != nullptr && bad_rows(v_rho_rows, n, out_rows)) ||
      !(viewmat_rows == 4 || viewmat_rows == 4 * B))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "project_bwd: operand rows must be n or B*n");
  if (fold_batch && (means3d_rows != n || scales_rows != n || quats_rows != n))
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "project_bwd: folded gradients need shared means, scales and quats");
  const int32_t K = num_transforms > 0 ? num_transforms : 1;
  if (has_transforms && !(transforms_rows == K || transforms_rows == K * B))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "project_bwd: transforms must have K or B*K matrices");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  {
    const ClearSpan spans[2] = {{v_viewmat, sizeof(float) * 16 * static_cast<size_t>(B)},
                                {v_transforms, sizeof(float) * 16 * static_cast<size_t>(K * B)}};
    launch_clear(spans, 2, stream);
  }
  ProjectBwdArgs a;
  a.means = means3d;
  a.scales = scales;
  a.quats = quats_xyzw;
  a.viewmat = viewmat;
  a.radii = radii;
  a.conics = conics;
  a.v_xy = v_xy;
  a.v_depth = v_depth;
  a.v_conic = v_conic;
  a.transforms = gaussian_transforms;
  a.transform_ids = transform_ids;
  a.n = n;
  a.B = B;
  a.num_transforms = K;
  a.has_transforms = has_transforms != 0;
  a.sel_means = means3d_rows > n;
  a.sel_scales = scales_rows > n;
  a.sel_quats = quats_rows > n;
  a.sel_view = viewmat_rows > 4;
  a.sel_radii = radii_rows > n;
  a.sel_conics = conics_rows > n;
  a.sel_vxy = v_xy_rows > n;
  a.sel_vdepth = v_depth_rows > n;
  a.sel_vconic = v_conic_rows > n;
  a.sel_transforms = transforms_rows > K;
  a.fx = fx;
  a.fy = fy;
  a.glob_scale = glob_scale;
  a.v_mean3d = v_mean3d;
  a.v_scale = v_scale;
  a.v_quat = v_quat;
  a.v_viewmat = v_viewmat;
  a.v_transforms = v_transforms;
  a.v_rho = v_rho;
  a.sel_vrho = v_rho_rows > n;
  a.aa_eps = aa_eps;
  a.aa_eps2 = aa_eps2;
  a.quats_wxyz = quats_wxyz != 0;
  a.fold_batch = fold_batch != 0;
  st->timer.begin(kProjectBwd, 1, stream);
  launch_project_bwd(a, stream);
  st->timer.end(stream);
  st->units.pairs_bwd += out_rows;
  return finish(*st, stream);
}

int splax_project_bwd(const float* means3d, int64_t means3d_rows, const float* scales,
                      int64_t scales_rows, const float* quats_xyzw, int64_t quats_rows,
                      const float* viewmat, int64_t viewmat_rows, const int32_t* radii,
                      int64_t radii_rows, const float* conics, int64_t conics_rows,
                      const float* v_xy, int64_t v_xy_rows, const float* v_depth,
                      int64_t v_depth_rows, const float* v_conic, int64_t v_conic_rows,
                      const float* gaussian_transforms, int64_t transforms_rows,
                      const int32_t* transform_ids, int32_t num_gaussians, int32_t num_transforms,
                      int32_t has_transforms, float fx, float fy, float glob_scale,
                      int64_t out_rows, float* v_mean3d, float* v_scale, float* v_quat,
                      float* v_viewmat, float* v_transforms, void* stream) {
  SPLAX_NVTX("splax_project_bwd");
  return project_bwd_impl(means3d, means3d_rows, scales, scales_rows, quats_xyzw, quats_rows,
                          viewmat, viewmat_rows, radii, radii_rows, conics, conics_rows, v_xy,
                          v_xy_rows, v_depth, v_depth_rows, v_conic, v_conic_rows, nullptr, 0,
                          0.0f, 0.0f, gaussian_transforms, transforms_rows, transform_ids,
                          num_gaussians, num_transforms, has_transforms, fx, fy, glob_scale,
                          out_rows, 0, 0, v_mean3d, v_scale, v_quat, v_viewmat, v_transforms,
                          stream);
}

int splax_project_bwd_ex(const float* means3d, int64_t means3d_rows, const float* scales,
                         int64_t scales_rows, const float* quats, int64_t quats_rows,
                         const float* viewmat, int64_t viewmat_rows, const int32_t* radii,
                         int64_t radii_rows, const float* conics, int64_t conics_rows,
                         const float* v_xy, int64_t v_xy_rows, const float* v_depth,
                         int64_t v_depth_rows, const float* v_conic, int64_t v_conic_rows,
                         const float* v_rho, int64_t v_rho_rows, float aa_eps, float aa_eps2,
                         const float* gaussian_transforms, int64_t transforms_rows,
                         const int32_t* transform_ids, int32_t num_gaussians,
                         int32_t num_transforms, int32_t has_transforms, float fx, float fy,
                         float glob_scale, int64_t out_rows, int32_t quats_wxyz,
                         int32_t fold_batch, float* v_mean3d, float* v_scale, float* v_quat,
                         float* v_viewmat, float* v_transforms, void* stream) {
  SPLAX_NVTX("splax_project_bwd_ex");
  return project_bwd_impl(means3d, means3d_rows, scales, scales_rows, quats, quats_rows,
                          viewmat, viewmat_rows, radii, radii_rows, conics, conics_rows, v_xy,
                          v_xy_rows, v_depth, v_depth_rows, v_conic, v_conic_rows, v_rho,
                          v_rho_rows, aa_eps, aa_eps2, gaussian_transforms, transforms_rows,
                          transform_ids, num_gaussians, num_transforms, has_transforms, fx, fy,
                          glob_scale, out_rows, quats_wxyz, fold_batch, v_mean3d, v_scale,
                          v_quat, v_viewmat, v_transforms, stream);
}

int splax_rasterize(const float* colors, int64_t colors_rows, const float* opacities,
                    int64_t opacities_rows, const float* map_opacities, int64_t map_opacities_rows,
                    const float* background, int64_t background_rows, const float* xys,
                    const float* depths, const int32_t* radii, const float* conics,
                    const int32_t* cum_tiles_hit, int64_t geom_rows, int32_t num_gaussians,
                    int32_t img_h, int32_t img_w, int64_t out_rows, int32_t key_bits,
                    float* final_Ts, int32_t* final_idx, float* out_img, void* stream) {
  SPLAX_NVTX("splax_rasterize");
  return rasterize_common(colors, colors_rows, opacities, opacities_rows, map_opacities,
                          map_opacities_rows, background, background_rows, xys, depths, radii,
                          conics, cum_tiles_hit, geom_rows, num_gaussians, img_h, img_w, out_rows,
                          key_bits, final_Ts, final_idx, out_img, nullptr,
                          static_cast<cudaStream_t>(stream));
}

int splax_rasterize_depth(const float* colors, int64_t colors_rows, const float* opacities,
                          int64_t opacities_rows, const float* map_opacities,
                          int64_t map_opacities_rows, const float* background,
                          int64_t background_rows, const float* xys, const float* depths,
                          const int32_t* radii, const float* conics, const int32_t* cum_tiles_hit,
                          int64_t geom_rows, int32_t num_gaussians, int32_t img_h, int32_t img_w,
                          int64_t out_rows, int32_t key_bits, float* final_Ts, int32_t* final_idx,
                          float* out_img, float* out_depth, void* stream) {
  SPLAX_NVTX("splax_rasterize_depth");
  if (!out_depth) return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize_depth: out_depth is NULL");
  return rasterize_common(colors, colors_rows, opacities, opacities_rows, map_opacities,
                          map_opacities_rows, background, background_rows, xys, depths, radii,
                          conics, cum_tiles_hit, geom_rows, num_gaussians, img_h, img_w, out_rows,
                          key_bits, final_Ts, final_idx, out_img, out_depth,
                          static_cast<cudaStream_t>(stream));
}

int splax_rasterize_bwd(const float* colors, int64_t colors_rows, const float* opacities,
                        int64_t opacities_rows, const float* map_opacities,
                        int64_t map_opacities_rows, const float* background,
                        int64_t background_rows, const float* xys, const float* depths,
                        const int32_t* radii, const float* conics, const int32_t* cum_tiles_hit,
                        int64_t geom_rows, const float* final_Ts, const int32_t* final_idx,
                        const float* v_out_img, int64_t v_out_rows, int32_t num_gaussians,
                        int32_t img_h, int32_t img_w, int64_t grad_rows, int32_t key_bits,
                        float* v_colors, float* v_opacity, float* v_xy, float* v_conic,
                        void* stream) {
  SPLAX_NVTX("splax_rasterize_bwd");
  return rasterize_bwd_common(colors, colors_rows, opacities, opacities_rows, map_opacities,
                              map_opacities_rows, background, background_rows, xys, depths,
                              radii, conics, cum_tiles_hit, geom_rows, final_Ts, final_idx,
                              v_out_img, v_out_rows, nullptr, 0, num_gaussians, img_h, img_w,
                              grad_rows, key_bits, v_colors, v_opacity, v_xy, v_conic, nullptr,
                              false, false, static_cast<cudaStream_t>(stream));
}

int splax_rasterize_bwd_depth(const float* colors, int64_t colors_rows, const float* opacities,
                              int64_t opacities_rows, const float* map_opacities,
                              int64_t map_opacities_rows, const float* background,
                              int64_t background_rows, const float* xys, const float* depths,
                              const int32_t* radii, const float* conics,
                              const int32_t* cum_tiles_hit, int64_t geom_rows,
                              const float* final_Ts, const int32_t* final_idx,
                              const float* v_out_img, int64_t v_out_rows,
                              const float* v_out_depth, int64_t v_out_depth_rows,
                              int32_t num_gaussians, int32_t img_h, int32_t img_w,
                              int64_t grad_rows, int32_t key_bits, float* v_colors,
                              float* v_opacity, float* v_xy, float* v_conic, float* v_depths,
                              void* stream) {
  SPLAX_NVTX("splax_rasterize_bwd_depth");
  if (!v_out_depth || !v_depths)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "rasterize_bwd_depth: depth buffers are NULL");
  return rasterize_bwd_common(colors, colors_rows, opacities, opacities_rows, map_opacities,
                              map_opacities_rows, background, background_rows, xys, depths,
                              radii, conics, cum_tiles_hit, geom_rows, final_Ts, final_idx,
                              v_out_img, v_out_rows, v_out_depth, v_out_depth_rows, num_gaussians,
                              img_h, img_w, grad_rows, key_bits, v_colors, v_opacity, v_xy,
                              v_conic, v_depths, false, false, static_cast<cudaStream_t>(stream));
}

int splax_rasterize_bwd_ex(const float* colors, int64_t colors_rows, const float* opacities,
                           int64_t opacities_rows, const float* map_opacities,
                           int64_t map_opacities_rows, const float* background,
                           int64_t background_rows, const float* xys, const float* depths,
                           const int32_t* radii, const float* conics,
                           const int32_t* cum_tiles_hit, int64_t geom_rows,
                           const float* final_Ts, const int32_t* final_idx,
                           const float* v_out_img, int64_t v_out_rows, const float* v_out_depth,
                           int64_t v_out_depth_rows, int32_t num_gaussians, int32_t img_h,
                           int32_t img_w, int64_t grad_rows, int32_t key_bits,
                           int32_t fold_colors, int32_t fold_opacity, float* v_colors,
                           float* v_opacity, float* v_xy, float* v_conic, float* v_depths,
                           void* stream) {
  SPLAX_NVTX("splax_rasterize_bwd_ex");
  if ((v_out_depth == nullptr) != (v_depths == nullptr))
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "rasterize_bwd_ex: v_out_depth and v_depths must be given together");
  return rasterize_bwd_common(colors, colors_rows, opacities, opacities_rows, map_opacities,
                              map_opacities_rows, background, background_rows, xys, depths,
                              radii, conics, cum_tiles_hit, geom_rows, final_Ts, final_idx,
                              v_out_img, v_out_rows, v_out_depth, v_out_depth_rows, num_gaussians,
                              img_h, img_w, grad_rows, key_bits, v_colors, v_opacity, v_xy,
                              v_conic, v_depths, fold_colors != 0, fold_opacity != 0,
                              static_cast<cudaStream_t>(stream));
}

int splax_sort_and_bin(const float* xys, const float* depths, const int32_t* radii,
                       const float* conics, const float* map_opacities,
                       int64_t map_opacities_rows, const int32_t* cum_tiles_hit,
                       int32_t num_gaussians, int32_t num_images, int32_t img_h, int32_t img_w,
                       int32_t key_bits, int32_t* gaussian_ids, int64_t gaussian_ids_cap,
                       int64_t* sorted_keys, int32_t* tile_bins, int64_t* num_intersects,
                       int32_t* used_key_bits, void* stream_) {
  SPLAX_NVTX("splax_sort_and_bin");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (num_gaussians <= 0 || num_images <= 0 || img_h <= 0 || img_w <= 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "sort_and_bin: invalid sizes");
  const int64_t total = static_cast<int64_t>(num_images) * num_gaussians;
  if (bad_rows(map_opacities_rows, num_gaussians, total))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "sort_and_bin: map_opacities rows must be n or B*n");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  // no colours: the blend records are not packed
  SortIn in{xys, depths, radii, conics, map_opacities, map_opacities_rows, nullptr, 1, nullptr, 1,
            cum_tiles_hit, num_gaussians, num_images, img_h, img_w, key_bits};
  SortOut so;
  rc = sort_and_bin(*st, in, stream, so);
  if (rc) return rc;
  if (so.count > gaussian_ids_cap)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "sort_and_bin: gaussian_ids capacity too small");
  if (so.count > 0) {
    SPLAX_CUDA(cudaMemcpyAsync(gaussian_ids, so.gids, sizeof(int32_t) * so.count,
                               cudaMemcpyDeviceToDevice, stream));
  }
  SPLAX_CUDA(cudaMemcpyAsync(tile_bins, so.bins,
                             sizeof(int2) * static_cast<int64_t>(num_images) * so.num_tiles,
                             cudaMemcpyDeviceToDevice, stream));
  if (sorted_keys && so.count > 0) {
    // the reference's own key for each sorted intersection
    PairKeyArgs pa;
    pa.depths = depths;
    pa.radii = radii;
    pa.depth_mm = so.depth_mm;
    pa.n = num_gaussians;
    pa.total = total;
    pa.packed = so.key_bits == 32;
    pa.depth_bits = so.depth_bits;
    pa.key_shift = 0;
    pa.err = st->err_word();
    pa.walk = nullptr;
    pa.records = nullptr;
    launch_reference_keys(so.keys, so.gids, so.count, pa, sorted_keys, stream);
  }
  *num_intersects = so.count;
  *used_key_bits = so.key_bits;
  return finish(*st, stream);
}

int splax_mse_loss(const float* img, const float* target, int64_t count, float denom,
                   float* loss, void* stream_) {
  SPLAX_NVTX("splax_mse_loss");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (count < 0 || !(denom > 0.0f) || loss == nullptr ||
      (count > 0 && (img == nullptr || target == nullptr)))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "mse_loss: invalid count, denom or pointers");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  const int blocks = mse_loss_blocks();
  const size_t need = sizeof(double) * (blocks + 1);
  if (st->loss.bytes < need) {
    SPLAX_CUDA(buf_reserve(st->loss, need));
    SPLAX_CUDA(cudaMemsetAsync(st->loss.p, 0, need, stream));
  }
  double* partials = static_cast<double*>(st->loss.p);
  st->timer.begin(kLoss, 1, stream);
  launch_mse_loss(img, target, count, 1.0 / static_cast<double>(denom), partials,
                  reinterpret_cast<unsigned*>(partials + blocks), loss, blocks, stream);
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_mse_loss_bwd(const float* img, const float* target, int64_t count, float denom,
                       const float* v_loss, float* grad, void* stream_) {
  SPLAX_NVTX("splax_mse_loss_bwd");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (count < 0 || !(denom > 0.0f) || v_loss == nullptr ||
      (count > 0 && (img == nullptr || target == nullptr || grad == nullptr)))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "mse_loss_bwd: invalid count, denom or pointers");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  st->timer.begin(kLoss, count > 0 ? 1 : 0, stream);
  if (count > 0)
    launch_mse_loss_bwd(img, target, count, 2.0f / denom, v_loss, grad, mse_loss_blocks(),
                        stream);
  st->timer.end(stream);
  return finish(*st, stream);
}

// The 11-tap Gaussian window of sigma 1.5, normalised, in fp32 (the window dm_pix.ssim builds).
static void ssim_window_weights(float* w) {
  float sum = 0.0f;
  for (int i = 0; i < 11; ++i) {
    const float t = (static_cast<float>(i) - 5.0f) / 1.5f;
    w[i] = std::exp(-0.5f * (t * t));
    sum += w[i];
  }
  for (int i = 0; i < 11; ++i) w[i] /= sum;
}

static int l1_dssim_check(const float* img, const float* target, int32_t B, int32_t H,
                          int32_t W, int32_t views_total, float ssim_lambda, const char* who) {
  if (B <= 0 || H < 11 || W < 11 || views_total < B || !(ssim_lambda >= 0.0f) ||
      !(ssim_lambda <= 1.0f) || img == nullptr || target == nullptr)
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                std::string(who) + ": need B >= 1, H, W >= 11, views_total >= B, lambda in [0, 1]");
  return SPLAX_OK;
}

int splax_l1_dssim_loss(const float* img, const float* target, int32_t B, int32_t H, int32_t W,
                        int32_t views_total, float ssim_lambda, float* loss, void* stream_) {
  SPLAX_NVTX("splax_l1_dssim_loss");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = l1_dssim_check(img, target, B, H, W, views_total, ssim_lambda, "l1_dssim_loss");
  if (rc) return rc;
  if (loss == nullptr) return fail(SPLAX_ERR_INVALID_ARGUMENT, "l1_dssim_loss: loss is NULL");
  DeviceState* st;
  rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  if (!st->ssim_window) {
    float w[11];
    ssim_window_weights(w);
    ssim_set_window(w);
    SPLAX_CUDA(cudaGetLastError());
    st->ssim_window = true;
  }
  SPLAX_CUDA(buf_reserve(st->ssim_partials, sizeof(double2) * l1_dssim_partials_max(B, H, W)));
  const double V = views_total, lam = ssim_lambda;
  const double l1_scale = (1.0 - lam) / (V * H * W * 3.0);
  const double ssim_scale = lam / (V * (H - 10.0) * (W - 10.0) * 3.0);
  st->timer.begin(kLoss, 2, stream);
  launch_l1_dssim(img, target, B, H, W, l1_scale, ssim_scale, lam * B / V,
                  static_cast<double2*>(st->ssim_partials.p), loss, stream);
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_l1_dssim_loss_bwd(const float* img, const float* target, int32_t B, int32_t H,
                            int32_t W, int32_t views_total, float ssim_lambda,
                            const float* v_loss, float* grad, void* stream_) {
  SPLAX_NVTX("splax_l1_dssim_loss_bwd");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = l1_dssim_check(img, target, B, H, W, views_total, ssim_lambda, "l1_dssim_loss_bwd");
  if (rc) return rc;
  if (v_loss == nullptr || grad == nullptr)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "l1_dssim_loss_bwd: v_loss or grad is NULL");
  DeviceState* st;
  rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  if (!st->ssim_window) {
    float w[11];
    ssim_window_weights(w);
    ssim_set_window(w);
    SPLAX_CUDA(cudaGetLastError());
    st->ssim_window = true;
  }
  const double V = views_total, lam = ssim_lambda;
  const float l1_scale = static_cast<float>((1.0 - lam) / (V * H * W * 3.0));
  const float ssim_grad = static_cast<float>(-lam / (V * (H - 10.0) * (W - 10.0) * 3.0));
  st->timer.begin(kLoss, 1, stream);
  launch_l1_dssim_bwd(img, target, B, H, W, l1_scale, ssim_grad, v_loss, grad, stream);
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_l1_dssim_loss_and_grad(const float* img, const float* target, int32_t B, int32_t H,
                                 int32_t W, int32_t views_total, float ssim_lambda, float* loss,
                                 float* grad, void* stream_) {
  SPLAX_NVTX("splax_l1_dssim_loss_and_grad");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int rc = l1_dssim_check(img, target, B, H, W, views_total, ssim_lambda,
                          "l1_dssim_loss_and_grad");
  if (rc) return rc;
  if (loss == nullptr || grad == nullptr)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "l1_dssim_loss_and_grad: loss or grad is NULL");
  DeviceState* st;
  rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  if (!st->ssim_window) {
    float w[11];
    ssim_window_weights(w);
    ssim_set_window(w);
    SPLAX_CUDA(cudaGetLastError());
    st->ssim_window = true;
  }
  SPLAX_CUDA(buf_reserve(st->ssim_partials, sizeof(double2) * l1_dssim_partials_max(B, H, W)));
  const double V = views_total, lam = ssim_lambda;
  const double l1_scale = (1.0 - lam) / (V * H * W * 3.0);
  const double ssim_scale = lam / (V * (H - 10.0) * (W - 10.0) * 3.0);
  st->timer.begin(kLoss, 2, stream);
  launch_l1_dssim_and_grad(img, target, B, H, W, l1_scale, ssim_scale, lam * B / V,
                           static_cast<float>(l1_scale), static_cast<float>(-ssim_scale),
                           static_cast<double2*>(st->ssim_partials.p), loss, grad, stream);
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_adam_step(int32_t num_arrays, float* const* params, const float* const* grads,
                    float* const* exp_avg, float* const* exp_avg_sq, const int64_t* sizes,
                    const float* lrs, int32_t step, float b1, float b2, float eps,
                    void* stream_) {
  SPLAX_NVTX("splax_adam_step");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (num_arrays < 0 || step < 1 || (num_arrays > 0 && (params == nullptr || grads == nullptr ||
                                                        exp_avg == nullptr ||
                                                        exp_avg_sq == nullptr ||
                                                        sizes == nullptr || lrs == nullptr)))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "adam_step: invalid arrays or step");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  // bias corrections as optax forms them in fp32: 1 - decay ** count
  const float bc1 = 1.0f - std::pow(b1, static_cast<float>(step));
  const float bc2 = 1.0f - std::pow(b2, static_cast<float>(step));
  for (int32_t j = 0; j < num_arrays; ++j)
    if (sizes[j] < 0 ||
        (sizes[j] > 0 && (!params[j] || !grads[j] || !exp_avg[j] || !exp_avg_sq[j])))
      return fail(SPLAX_ERR_INVALID_ARGUMENT, "adam_step: NULL array or negative size");
  st->timer.begin(kOptim, (num_arrays + kAdamMaxSegs - 1) / kAdamMaxSegs, stream);
  for (int32_t k0 = 0; k0 < num_arrays; k0 += kAdamMaxSegs) {
    AdamSegs s{};
    const int32_t cnt = num_arrays - k0 < kAdamMaxSegs ? num_arrays - k0 : kAdamMaxSegs;
    for (int32_t k = 0; k < cnt; ++k) {
      const int32_t j = k0 + k;
      s.seg[k] = AdamSeg{params[j], grads[j], exp_avg[j], exp_avg_sq[j], sizes[j], lrs[j]};
    }
    launch_adam(s, cnt, b1, b2, bc1, bc2, eps, stream);
  }
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_nvls_allreduce_f32(float* multicast, void* const* flag_ptrs, int32_t rank,
                             int32_t world, int64_t n, uint64_t epoch, uint32_t* err,
                             void* stream_) {
  SPLAX_NVTX("splax_nvls_allreduce_f32");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (multicast == nullptr || flag_ptrs == nullptr || err == nullptr || world < 1 ||
      world > 8 || rank < 0 || rank >= world || n < 0 || epoch == 0 ||
      reinterpret_cast<uintptr_t>(multicast) % 16 != 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "nvls_allreduce: NULL pointer, rank / world out of range, n < 0, epoch 0 or a "
                "multicast address not 16-byte aligned");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  auto* const* flags = reinterpret_cast<unsigned long long* const*>(flag_ptrs);
  st->timer.begin(kAllReduce, 3, stream);
  if (launch_nvls_barrier(flags, rank, world, epoch, err, stream) ||
      launch_nvls_allreduce(multicast, n, rank, world, err, stream) ||
      launch_nvls_barrier(flags, rank, world, epoch + 1, err, stream)) {
    st->timer.end(stream);
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "nvls_allreduce: invalid flag array");
  }
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_nvls_adam_shard_len(int64_t n, int32_t rank, int32_t world, int64_t* len) {
  if (len == nullptr || n < 0 || world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "nvls_adam_shard_len: invalid n, rank or world");
  *len = nvls_adam_shard_len(n, rank, world);
  return SPLAX_OK;
}

int splax_nvls_adam_step(const float* grad_mc, float* param_mc, const float* param_local,
                         float* exp_avg, float* exp_avg_sq, int64_t n, int32_t num_groups,
                         const int64_t* group_sizes, const float* lrs, int32_t step, float b1,
                         float b2, float eps, void* const* flag_ptrs, int32_t rank,
                         int32_t world, uint64_t epoch, uint32_t* err, void* stream_) {
  SPLAX_NVTX("splax_nvls_adam_step");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (grad_mc == nullptr || param_mc == nullptr || param_local == nullptr || exp_avg == nullptr ||
      exp_avg_sq == nullptr || group_sizes == nullptr || lrs == nullptr ||
      flag_ptrs == nullptr || err == nullptr || n < 0 || num_groups < 1 ||
      num_groups > kAdamMaxSegs || step < 1 || world < 1 || world > 8 || rank < 0 ||
      rank >= world || epoch == 0)
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "nvls_adam_step: NULL pointer, groups outside 1..8, step < 1, rank / world out "
                "of range or epoch 0");
  NvlsAdamGroups gr{};
  int64_t end = 0;
  for (int32_t k = 0; k < num_groups; ++k) {
    if (group_sizes[k] < 0)
      return fail(SPLAX_ERR_INVALID_ARGUMENT, "nvls_adam_step: negative group size");
    end += group_sizes[k];
    gr.end[k] = end;
    gr.lr[k] = lrs[k];
  }
  gr.count = num_groups;
  if (end != n)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "nvls_adam_step: group sizes do not add up to n");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  // bias corrections as optax forms them in fp32 (as splax_adam_step)
  const float bc1 = 1.0f - std::pow(b1, static_cast<float>(step));
  const float bc2 = 1.0f - std::pow(b2, static_cast<float>(step));
  auto* const* flags = reinterpret_cast<unsigned long long* const*>(flag_ptrs);
  st->timer.begin(kAllReduce, 3, stream);
  if (launch_nvls_barrier(flags, rank, world, epoch, err, stream) ||
      launch_nvls_adam(grad_mc, param_mc, param_local, exp_avg, exp_avg_sq, n, rank, world, gr,
                       b1, b2, bc1, bc2, eps, err, stream) ||
      launch_nvls_barrier(flags, rank, world, epoch + 1, err, stream)) {
    st->timer.end(stream);
    return fail(SPLAX_ERR_INVALID_ARGUMENT,
                "nvls_adam_step: invalid flag array or a buffer not 16-byte aligned");
  }
  st->timer.end(stream);
  return finish(*st, stream);
}

int splax_ply_info(const char* path, int64_t* num_vertices) {
  if (path == nullptr || num_vertices == nullptr)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "ply_info: NULL argument");
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(SPLAX_ERR_INVALID_ARGUMENT, std::string("ply_info: cannot open ") + path);
  PlyLayout L;
  int64_t n = 0, body = 0;
  std::string why;
  const int rc = ply_parse_header(f, &L, &n, &body, &why);
  std::fclose(f);
  if (rc) return fail(SPLAX_ERR_INVALID_ARGUMENT, "ply_info: " + why);
  *num_vertices = n;
  return SPLAX_OK;
}

int splax_ply_load(const char* path, int64_t num_vertices, float* means, float* scales,
                   float* quats, float* colors, float* opacities, void* stream_) {
  SPLAX_NVTX("splax_ply_load");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (path == nullptr || num_vertices < 0 ||
      (num_vertices > 0 && (!means || !scales || !quats || !colors || !opacities)))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "ply_load: invalid arguments");
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(SPLAX_ERR_INVALID_ARGUMENT, std::string("ply_load: cannot open ") + path);
  struct Closer {
    FILE* f;
    ~Closer() { std::fclose(f); }
  } closer{f};
  PlyLayout L;
  int64_t n = 0, body = 0;
  std::string why;
  if (ply_parse_header(f, &L, &n, &body, &why))
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "ply_load: " + why);
  if (n != num_vertices)
    return fail(SPLAX_ERR_INVALID_ARGUMENT, "ply_load: num_vertices does not match the file");
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  constexpr size_t kChunk = size_t(32) << 20;
  const size_t chunk = std::max<size_t>(kChunk, static_cast<size_t>(L.stride));
  if (st->ply_chunk < chunk) {
    SPLAX_CUDA(cudaStreamSynchronize(stream));
    for (int b = 0; b < 2; ++b) {
      if (st->ply_host[b]) cudaFreeHost(st->ply_host[b]);
      st->ply_host[b] = nullptr;
      buf_free(st->ply_dev[b]);
    }
    st->ply_chunk = 0;
    for (int b = 0; b < 2; ++b) {
      SPLAX_CUDA(cudaMallocHost(&st->ply_host[b], chunk));
      SPLAX_CUDA(buf_reserve(st->ply_dev[b], chunk));
      if (!st->ply_ev[b]) SPLAX_CUDA(cudaEventCreateWithFlags(&st->ply_ev[b], cudaEventDisableTiming));
    }
    st->ply_chunk = chunk;
  }
  const int64_t per = static_cast<int64_t>(chunk / static_cast<size_t>(L.stride));
  int b = 0;
  for (int64_t first = 0; first < n; first += per, b ^= 1) {
    const int64_t cnt = std::min<int64_t>(per, n - first);
    const size_t bytes = static_cast<size_t>(cnt * L.stride);
    SPLAX_CUDA(cudaEventSynchronize(st->ply_ev[b]));  // the copy out of this buffer is done
    if (std::fread(st->ply_host[b], 1, bytes, f) != bytes)
      return fail(SPLAX_ERR_INVALID_ARGUMENT, "ply_load: the file is shorter than its header says");
    SPLAX_CUDA(cudaMemcpyAsync(st->ply_dev[b].p, st->ply_host[b], bytes, cudaMemcpyHostToDevice,
                               stream));
    SPLAX_CUDA(cudaEventRecord(st->ply_ev[b], stream));
    launch_ply_decode(static_cast<const unsigned char*>(st->ply_dev[b].p), cnt, L, first, means,
                      scales, quats, colors, opacities, stream);
  }
  return finish(*st, stream);
}

void splax_clear_cache(void) {
  std::lock_guard<std::mutex> lk(g_states_mu);
  int prev = 0;
  cudaGetDevice(&prev);
  for (auto& s : g_states) {
    if (!s) continue;
    std::lock_guard<std::mutex> lk2(s->mu);
    if (cudaSetDevice(s->device) != cudaSuccess) continue;
    cudaDeviceSynchronize();
    s->drop_entry();
  }
  cudaSetDevice(prev);
}

int splax_scratch_info(int64_t* out, int32_t out_len) {
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return -rc;
  std::lock_guard<std::mutex> lk(st->mu);
  const int64_t vals[6] = {st->isect_cap, st->key_bits, static_cast<int64_t>(st->bytes_held()),
                           st->sig_B, st->sig_n, st->sig_T};
  int k = 0;
  for (; k < out_len && k < 6; ++k) out[k] = vals[k];
  return k;
}

int splax_check_device_errors(void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  if (!st->ev) return SPLAX_OK;
  SPLAX_CUDA(cudaStreamSynchronize(stream));
  unsigned w = 0;
  SPLAX_CUDA(cudaMemcpy(&w, st->err_word(), sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (w) return report_device_error(*st, w, stream);
  return SPLAX_OK;
}

void splax_debug_fail_alloc_after(int64_t successes) { g_fail_after.store(successes); }

int64_t splax_last_sort_token(void) { return g_last_sort_token; }

void splax_reuse_sort(int64_t token) { g_armed_sort_token = token; }

void splax_profile_enable(int32_t timing, int32_t count_work) {
  g_timing.store(timing != 0);
  g_count_work.store(count_work != 0);
}

void splax_profile_stages(uint32_t mask) { g_timing_mask.store(mask); }

int splax_profile_reset(void) {
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return rc;
  st->timer.reset();
  st->units = WorkUnits{};
  SPLAX_CUDA(cudaMemset(st->work.p, 0, kWorkWords * sizeof(unsigned long long)));
  return SPLAX_OK;
}

int splax_profile_report(char* buf, int32_t len) {
  DeviceState* st;
  int rc = current_state(&st);
  if (rc) return -rc;
  std::lock_guard<std::mutex> lk(st->mu);
  rc = st->init();
  if (rc) return -rc;
  st->timer.collect();
  unsigned long long w[kWorkWords] = {};
  if (cudaMemcpy(w, st->work.p, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess) return -SPLAX_ERR_CUDA;
  std::string js = "{\"kernels\": {";
  char tmp[256];
  for (int k = 0; k < kNumKinds; ++k) {
    snprintf(tmp, sizeof tmp, "%s\"%s\": {\"launches\": %lld, \"kernels\": %lld, \"ms\": %.6f}",
             k ? ", " : "", kKindNames[k], static_cast<long long>(st->timer.launches[k]),
             static_cast<long long>(st->timer.kernels[k]), st->timer.ms[k]);
    js += tmp;
  }
  const WorkUnits& u = st->units;
  snprintf(tmp, sizeof tmp,
           "}, \"units\": {\"pairs_fwd\": %lld, \"pairs_bwd\": %lld, \"intersections\": %lld, "
           "\"key_bytes\": %lld, \"sort_pass_keys\": %lld, \"bins\": %lld, ",
           (long long)u.pairs_fwd, (long long)u.pairs_bwd, (long long)u.intersections,
           (long long)u.key_bytes, (long long)u.sort_passes, (long long)u.bins);
  js += tmp;
  snprintf(tmp, sizeof tmp,
           "\"pixels_fwd\": %lld, \"pixels_bwd\": %lld, \"fwd_evals\": %llu, "
           "\"fwd_contribs\": %llu, \"bwd_evals\": %llu, \"bwd_contribs\": %llu, "
           "\"sort_reuses\": %lld, ",
           (long long)u.pixels_fwd, (long long)u.pixels_bwd, w[0], w[1], w[2], w[3],
           (long long)u.sort_reuses);
  js += tmp;
  snprintf(tmp, sizeof tmp,
           "\"pairs_sorted\": %lld, \"pair_key_bytes\": %lld, \"pair_pass_keys\": %lld, ",
           (long long)u.pairs_sorted, (long long)u.pair_key_bytes, (long long)u.pair_pass_keys);
  js += tmp;
  snprintf(tmp, sizeof tmp,
           "\"bwd_warp_steps\": %llu, \"bwd_warp_steps_active\": %llu}}", w[4], w[5]);
  js += tmp;
  if (static_cast<int32_t>(js.size()) + 1 > len) return -SPLAX_ERR_INVALID_ARGUMENT;
  memcpy(buf, js.c_str(), js.size() + 1);
  return static_cast<int>(js.size());
}

}  // extern "C"
