// Projection forward (tile count + fused global scan) and projection backward.
//
// Forward: one thread per (camera, gaussian) pair of the flat B*N launch, the work of
// _project_kernel (splax/_project/_kernels.py:122-248) followed by the global inclusive scan
// (:104-107) done in the same kernel with a decoupled look-back, so num_tiles_hit is never
// re-read. Compiled with --fmad=false: every float op rounds as written, which makes the
// integer outputs (radii, tile counts, cum) bit-identical to the C oracle.
//
// Backward: _project_bwd_kernel (:356-484) with its vjp helpers (:487-664); the per-image
// viewmat cotangent is reduced per block with a warp reduce-scatter before one atomic per
// entry per block.
#include "common.cuh"
#include "kernels.h"

namespace splax {
namespace {

__device__ __forceinline__ void mat_mul(const float* A, const float* B, float* C) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      C[3 * i + j] = (A[3 * i] * B[j] + A[3 * i + 1] * B[3 + j]) + A[3 * i + 2] * B[6 + j];
}
__device__ __forceinline__ void mat_T(const float* A, float* C) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) C[3 * i + j] = A[3 * j + i];
}
__device__ __forceinline__ void mat_vec(const float* A, const float* v, float* o) {
#pragma unroll
  for (int i = 0; i < 3; ++i) o[i] = (A[3 * i] * v[0] + A[3 * i + 1] * v[1]) + A[3 * i + 2] * v[2];
}
// rows r..r+2 of a (rows, 4) row-major matrix (_load_affine, :609-624)
__device__ __forceinline__ void load_affine(const float* m, float* R, float* t) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    R[3 * i] = m[4 * i];
    R[3 * i + 1] = m[4 * i + 1];
    R[3 * i + 2] = m[4 * i + 2];
    t[i] = m[4 * i + 3];
  }
}
// rotation of a unit xyzw quaternion; its derivative is _quat_vjp (:570-599)
__device__ __forceinline__ void quat_to_mat(float x, float y, float z, float w, float* R) {
  R[0] = 1.0f - 2.0f * (y * y + z * z);
  R[1] = 2.0f * (x * y - w * z);
  R[2] = 2.0f * (x * z + w * y);
  R[3] = 2.0f * (x * y + w * z);
  R[4] = 1.0f - 2.0f * (x * x + z * z);
  R[5] = 2.0f * (y * z - w * x);
  R[6] = 2.0f * (x * z - w * y);
  R[7] = 2.0f * (y * z + w * x);
  R[8] = 1.0f - 2.0f * (x * x + y * y);
}

struct Geom {
  float W[9], p[3], M[9], R_tf[9], mean[3];
  bool moved;
};

// _apply_transform + _project_geom (:627-664)
__device__ __forceinline__ void project_geom(const ProjectArgs& a, int64_t idx, int64_t bid,
                                             int64_t gid, Geom& g, float* q, float* sc) {
  int64_t m_idx = a.sel_means ? idx : gid;
  int64_t s_idx = a.sel_scales ? idx : gid;
  int64_t q_idx = a.sel_quats ? idx : gid;
  int64_t vb = (a.sel_view ? bid : 0) * 4;
  g.mean[0] = a.means[3 * m_idx];
  g.mean[1] = a.means[3 * m_idx + 1];
  g.mean[2] = a.means[3 * m_idx + 2];
  // q = (x, y, z, w); wxyz storage (the public API's order) is read without a reorder pass
  const int qo = a.quats_wxyz ? 1 : 0;
  q[0] = a.quats[4 * q_idx + qo];
  q[1] = a.quats[4 * q_idx + qo + 1];
  q[2] = a.quats[4 * q_idx + qo + 2];
  q[3] = a.quats[4 * q_idx + (a.quats_wxyz ? 0 : 3)];
  sc[0] = a.scales[3 * s_idx];
  sc[1] = a.scales[3 * s_idx + 1];
  sc[2] = a.scales[3 * s_idx + 2];
#pragma unroll
  for (int i = 0; i < 9; ++i) g.R_tf[i] = (i % 4 == 0) ? 1.0f : 0.0f;
  g.moved = false;
  int32_t tf_id = a.has_transforms ? a.transform_ids[gid] : -1;
  if (tf_id >= a.num_transforms) tf_id = -1;  // out-of-range ids are treated as static
  if (tf_id >= 0) {
    int64_t tf_idx = a.sel_transforms ? bid * a.num_transforms + tf_id : tf_id;
    float t[3], o[3];
    load_affine(a.transforms + tf_idx * 16, g.R_tf, t);
    mat_vec(g.R_tf, g.mean, o);
#pragma unroll
    for (int i = 0; i < 3; ++i) g.mean[i] = o[i] + t[i];
    g.moved = true;
  }
  float trans[3], Wm[3];
  load_affine(a.viewmat + vb * 4, g.W, trans);
  mat_vec(g.W, g.mean, Wm);
#pragma unroll
  for (int i = 0; i < 3; ++i) g.p[i] = Wm[i] + trans[i];
  float R[9];
  quat_to_mat(q[0], q[1], q[2], q[3], R);
  float s[3] = {a.glob_scale * sc[0], a.glob_scale * sc[1], a.glob_scale * sc[2]};
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) g.M[3 * i + j] = R[3 * i + j] * s[j];
  if (g.moved) {
    float Mt[9];
    mat_mul(g.R_tf, g.M, Mt);
#pragma unroll
    for (int i = 0; i < 9; ++i) g.M[i] = Mt[i];
  }
}

// Mip-Splatting opacity compensation of a dilated conic (splax/_project/_project.py:95-117),
// one IEEE operation per step in the order of the reference's expression; eps2 is eps^2 as
// the caller rounds it. rho2 outside [0, 1] clamps (NaN propagates).
__device__ __forceinline__ float aa_rho2(float a, float b, float c, float eps, float eps2) {
  const float t3 = 1.0f - eps * (a + c);
  const float t7 = eps2 * (a * c - b * b);
  return t3 + t7;
}
__device__ __forceinline__ float aa_rho(float a, float b, float c, float eps, float eps2) {
  float r2 = aa_rho2(a, b, c, eps, eps2);
  r2 = r2 < 0.0f ? 0.0f : (r2 > 1.0f ? 1.0f : r2);
  return sqrtf(r2);
}

// Projection of one pair up to its tile count: writes the culled (zero) outputs, and for a pair
// that passes every cull returns true with its outputs in o and its ellipse walk in e (the count
// is taken warp-cooperatively by the caller, then project_store writes the outputs).
struct PairOut {
  float cx, cy, ca, cb, cc, depth, rho;
  int32_t radius;
};

template <bool AA>
__device__ __forceinline__ bool project_setup(const ProjectArgs& a, int64_t idx, PairOut& o,
                                              Ellipse& e) {
  int64_t bid = idx / a.n, gid = idx % a.n;
  a.xys[2 * idx] = 0.0f;
  a.xys[2 * idx + 1] = 0.0f;
  a.depths[idx] = 0.0f;
  a.radii[idx] = 0;
  a.conics[3 * idx] = 0.0f;
  a.conics[3 * idx + 1] = 0.0f;
  a.conics[3 * idx + 2] = 0.0f;
  a.num_tiles_hit[idx] = 0;
  if constexpr (AA) a.rho[idx] = 1.0f;
  Geom g;
  float q[4], sc[3];
  project_geom(a, idx, bid, gid, g, q, sc);
  if (g.p[2] <= a.clip_thresh) return false;
  float Mt[9], V3[9];
  mat_T(g.M, Mt);
  mat_mul(g.M, Mt, V3);
  // EWA projection of the covariance (:188-212)
  float tan_fovx = 0.5f * static_cast<float>(a.img_w) / a.fx;
  float tan_fovy = 0.5f * static_cast<float>(a.img_h) / a.fy;
  float lim_x = 1.3f * tan_fovx, lim_y = 1.3f * tan_fovy;
  float tx = g.p[0], ty = g.p[1], tz = g.p[2];
  tx = tz * fmin_w(lim_x, fmax_w(-lim_x, tx / tz));
  ty = tz * fmin_w(lim_y, fmax_w(-lim_y, ty / tz));
  float rz = 1.0f / tz;
  float rz2 = rz * rz;
  float J[9] = {a.fx * rz, 0.0f, (-a.fx * tx) * rz2, 0.0f, a.fy * rz, (-a.fy * ty) * rz2,
                0.0f, 0.0f, 0.0f};
  float T[9], TV[9];
  mat_mul(J, g.W, T);
  mat_mul(T, V3, TV);
  float c00 = (TV[0] * T[0] + TV[1] * T[1]) + TV[2] * T[2];
  float c01 = (TV[0] * T[3] + TV[1] * T[4]) + TV[2] * T[5];
  float c11 = (TV[3] * T[3] + TV[4] * T[4]) + TV[5] * T[5];
  float cxx = c00 + 0.3f, cxy = c01, cyy = c11 + 0.3f;
  float det = cxx * cyy - cxy * cxy;
  if (det == 0.0f) return false;
  float inv_det = 1.0f / det;
  float ca = cyy * inv_det, cb = -cxy * inv_det, cc = cxx * inv_det;
  float rw = 1.0f / (g.p[2] + 1e-6f);
  float center_x = (g.p[0] * rw) * a.fx + a.cx;
  float center_y = (g.p[1] * rw) * a.fy + a.cy;
  int32_t tbx = (a.img_w + kBlockWidth - 1) / kBlockWidth;
  int32_t tby = (a.img_h + kBlockWidth - 1) / kBlockWidth;
  float opac = a.opacities[a.sel_opac ? idx : gid];
  if (opac < kAlphaThreshold) return false;
  float t = iso_level(opac);
  float ext = sqrtf(t);
  float radius_x = ceilf(ext * sqrtf(cxx));
  float radius_y = ceilf(ext * sqrtf(cyy));
  if (radius_x <= 0.0f && radius_y <= 0.0f) return false;
  if (center_x + radius_x <= 0.0f || center_x - radius_x >= static_cast<float>(a.img_w) ||
      center_y + radius_y <= 0.0f || center_y - radius_y >= static_cast<float>(a.img_h))
    return false;
  ellipse_init(ca, cb, cc, t, center_x, center_y, tbx, tby, e);
  o.cx = center_x;
  o.cy = center_y;
  o.ca = ca;
  o.cb = cb;
  o.cc = cc;
  o.depth = g.p[2];
  o.radius = f2i(fmax_w(radius_x, radius_y));
  if constexpr (AA) o.rho = aa_rho(ca, cb, cc, a.aa_eps, a.aa_eps2);
  return true;
}

template <bool AA>
__device__ __forceinline__ void project_store(const ProjectArgs& a, int64_t idx, const PairOut& o,
                                              int32_t count) {
  a.num_tiles_hit[idx] = count;
  a.depths[idx] = o.depth;
  a.radii[idx] = o.radius;
  a.xys[2 * idx] = o.cx;
  a.xys[2 * idx + 1] = o.cy;
  a.conics[3 * idx] = o.ca;
  a.conics[3 * idx + 1] = o.cb;
  a.conics[3 * idx + 2] = o.cc;
  if constexpr (AA) a.rho[idx] = o.rho;
}

constexpr int kProjThreads = 256;
constexpr int kProjItems = kProjScanTile / kProjThreads;  // pairs per thread
constexpr int kProjTile = kProjScanTile;

// four CTAs per SM (64 registers, no spills): 0.42 ms per step vs 0.46 at the compiler's 69
template <bool AA>
__global__ void __launch_bounds__(kProjThreads, 4)
project_fwd_kernel(ProjectArgs a, unsigned long long* status, int* ticket, unsigned* err) {
  pdl_enter();
  __shared__ int s_tile;
  __shared__ __align__(16) int32_t s_cnt[kProjTile];
  __shared__ long long s_warp[kProjThreads / 32];
  __shared__ long long s_prefix;
  __shared__ WarpWalk s_walk[kProjThreads / 32];
  __shared__ int32_t s_wcnt[kProjThreads / 32][32];
  if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t base = tile * kProjTile;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int k = 0; k < kProjItems; ++k) {
    const int64_t idx = base + k * kProjThreads + tid;
    PairOut o;
    Ellipse e{};
    const bool live = idx < a.total && project_setup<AA>(a, idx, o, e);
    if (!live) e.valid = false;
    // the tile count of the warp's 32 pairs, row by row across the lanes: the sum of
    // ellipse_column's (mx - mn), as ellipse_tile_count takes it
    s_wcnt[warp][lane] = 0;
    int rexc;
    const int rows = warp_walk_share(s_walk[warp], lane, e, rexc);
    for (int c0 = 0; c0 < rows; c0 += 32) {
      int ow, u;
      int32_t mn, mx;
      warp_walk_row(s_walk[warp], lane, rexc, c0 + lane, rows, ow, u, mn, mx);
      if (c0 + lane < rows) atomicAdd(&s_wcnt[warp][ow], mx - mn);
    }
    __syncwarp();
    const int32_t count = live ? s_wcnt[warp][lane] : 0;
    __syncwarp();  // the shared walk is reused by the next item
    if (count > 0) project_store<AA>(a, idx, o, count);
    s_cnt[k * kProjThreads + tid] = count > 0 ? count : 0;
  }
  __syncthreads();
  // each thread scans 4 consecutive pairs; a block scan of the thread sums places them
  static_assert(kProjItems == 4, "the scan reads each thread's counts as one int4");
  const int4 c4 = reinterpret_cast<const int4*>(s_cnt)[tid];
  const int32_t c[kProjItems] = {c4.x, c4.y, c4.z, c4.w};
  const long long tsum = static_cast<long long>(c4.x) + c4.y + c4.z + c4.w;
  long long v = tsum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  long long wpre = 0, agg = 0;
#pragma unroll
  for (int w = 0; w < kProjThreads / 32; ++w) {
    if (w < warp) wpre += s_warp[w];
    agg += s_warp[w];
  }
  if (warp == 0) {
    long long prefix = 0;
    if (tile == 0) {
      if (lane == 0) st_relaxed(&status[0], kLookbackInc | static_cast<unsigned long long>(agg));
    } else {
      if (lane == 0) st_relaxed(&status[tile], kLookbackAgg | static_cast<unsigned long long>(agg));
      prefix = warp_lookback(status, tile, err);
      if (lane == 0)
        st_relaxed(&status[tile], kLookbackInc | static_cast<unsigned long long>(prefix + agg));
    }
    if (lane == 0) {
      s_prefix = prefix;
      if (base + kProjTile >= a.total && prefix + agg > 0x7fffffffll)
        atomicOr(err, kErrCountOverflow);
    }
  }
  __syncthreads();
  long long run = s_prefix + wpre + v - tsum;
#pragma unroll
  for (int m = 0; m < kProjItems; ++m) {
    run += c[m];
    const int64_t idx = base + tid * kProjItems + m;
    if (idx < a.total) a.cum_tiles_hit[idx] = static_cast<int32_t>(static_cast<uint32_t>(run));
  }
}

// ------------------------------------------------------------------ backward

constexpr int kBwdThreads = 256;
// three CTAs per SM (80 registers, a few spilled to L1): 0.295 ms per step vs 0.315 at two
// (126 registers) and 0.333 at four

// FOLD: one thread per gaussian, looping over the B images and summing the gaussian's
// cotangents over them in registers (means, scales and quats shared by the images: the sum
// the caller would otherwise take over B*n rows). Otherwise one thread per (image, gaussian).
template <bool AA, bool FOLD>
__global__ void __launch_bounds__(kBwdThreads, 3) project_bwd_kernel(ProjectBwdArgs a) {
  pdl_enter();
  const int64_t blocks_per_image = (a.n + kBwdThreads - 1) / kBwdThreads;
  const int64_t img0 = FOLD ? 0 : blockIdx.x / blocks_per_image;
  const int64_t img1 = FOLD ? a.B : img0 + 1;
  const int64_t gid = (FOLD ? blockIdx.x : blockIdx.x % blocks_per_image) * kBwdThreads +
                      threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc_mean[3] = {0.0f, 0.0f, 0.0f}, acc_scale[3] = {0.0f, 0.0f, 0.0f};
  float acc_quat[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int64_t image_id = img0; image_id < img1; ++image_id) {
  const int64_t idx = image_id * a.n + gid;
  // 12 viewmat entries, then 12 transform entries
  float vv[12];
#pragma unroll
  for (int k = 0; k < 12; ++k) vv[k] = 0.0f;
  float vtf[12];
#pragma unroll
  for (int k = 0; k < 12; ++k) vtf[k] = 0.0f;
  int32_t tf_id = -1;
  bool live = false;
  if (gid < a.n) {
    tf_id = a.has_transforms ? a.transform_ids[gid] : -1;
    if (tf_id >= a.num_transforms) tf_id = -1;
    live = a.radii[a.sel_radii ? idx : gid] > 0;
  }
  bool moved = false;
  if (live) {
    ProjectArgs pa;
    pa.means = a.means; pa.scales = a.scales; pa.quats = a.quats; pa.viewmat = a.viewmat;
    pa.transforms = a.transforms; pa.transform_ids = a.transform_ids;
    pa.n = a.n; pa.num_transforms = a.num_transforms; pa.has_transforms = a.has_transforms;
    pa.sel_means = a.sel_means; pa.sel_scales = a.sel_scales; pa.sel_quats = a.sel_quats;
    pa.sel_view = a.sel_view; pa.sel_transforms = a.sel_transforms;
    pa.quats_wxyz = a.quats_wxyz;
    pa.glob_scale = a.glob_scale;
    Geom g;
    float q[4], sc[3];
    project_geom(pa, idx, image_id, gid, g, q, sc);
    const float fx = a.fx, fy = a.fy, gs = a.glob_scale;
    moved = g.moved;
    float Mt[9], V[9], R[9];
    mat_T(g.M, Mt);
    mat_mul(g.M, Mt, V);
    quat_to_mat(q[0], q[1], q[2], q[3], R);
    float s[3] = {gs * sc[0], gs * sc[1], gs * sc[2]};
    const float* p = g.p;
    float rz = 1.0f / p[2];
    float rz2 = rz * rz;
    float J[9] = {fx * rz, 0.0f, (-fx * p[0]) * rz2, 0.0f, fy * rz, (-fy * p[1]) * rz2,
                  0.0f, 0.0f, 0.0f};
    float T[9];
    mat_mul(J, g.W, T);
    const int64_t c_idx = a.sel_conics ? idx : gid;
    const int64_t vc_idx = a.sel_vconic ? idx : gid;
    const int64_t vx_idx = a.sel_vxy ? idx : gid;
    const int64_t vd_idx = a.sel_vdepth ? idx : gid;
    const float* conic = a.conics + 3 * c_idx;
    const float* vcon = a.v_conic + 3 * vc_idx;
    float X0 = conic[0], X1 = conic[1], X3 = conic[2];
    float G0 = vcon[0], G1 = vcon[1], G3 = vcon[2];
    if constexpr (AA) {
      // rho = sqrt(clip(rho2, 0, 1)): d rho / d rho2 = 1 / (2 rho) inside [0, 1], else 0;
      // d rho2 / d(a, b, c) = (-eps + eps^2 c, -2 eps^2 b, -eps + eps^2 a)
      const float vr = a.v_rho[a.sel_vrho ? idx : gid];
      const float r2 = aa_rho2(X0, X1, X3, a.aa_eps, a.aa_eps2);
      if (r2 >= 0.0f && r2 <= 1.0f) {
        const float d = vr / (2.0f * sqrtf(r2));
        G0 += d * (a.aa_eps2 * X3 - a.aa_eps);
        G1 += d * (-2.0f * a.aa_eps2 * X1);
        G3 += d * (a.aa_eps2 * X0 - a.aa_eps);
      }
    }
    G1 = 0.5f * G1;
    float XG0 = X0 * G0 + X1 * G1, XG1 = X0 * G1 + X1 * G3;
    float XG2 = X1 * G0 + X3 * G1, XG3 = X1 * G1 + X3 * G3;
    float S0 = XG0 * X0 + XG1 * X1, S1 = XG0 * X1 + XG1 * X3;
    float S2 = XG2 * X0 + XG3 * X1, S3 = XG2 * X1 + XG3 * X3;
    float vc0 = -S0, vc1 = -(S1 + S2), vc2 = -S3;
    // _proj_vjp (:487-533)
    const float vx0 = a.v_xy ? a.v_xy[2 * vx_idx] : 0.0f;
    const float vx1 = a.v_xy ? a.v_xy[2 * vx_idx + 1] : 0.0f;
    const float vdep = a.v_depth ? a.v_depth[vd_idx] : 0.0f;
    float tx = p[0], ty = p[1], tz = p[2];
    float rz3 = rz2 * rz;
    float rw = 1.0f / (tz + 1e-6f);
    float vpx = fx * vx0, vpy = fy * vx1;
    float vvx = vpx * rw, vvy = vpy * rw;
    float vvz = (-(vpx * tx + vpy * ty) * rw) * rw + vdep;
    float vcov[9] = {vc0, 0.5f * vc1, 0.0f, 0.5f * vc1, vc2, 0.0f, 0.0f, 0.0f, 0.0f};
    float Tt[9], tmp[9], v_V[9], v_T[9], Wt[9], v_J[9], vc2m[9];
    mat_T(T, Tt);
    mat_mul(Tt, vcov, tmp);
    mat_mul(tmp, T, v_V);
#pragma unroll
    for (int k = 0; k < 9; ++k) vc2m[k] = 2.0f * vcov[k];
    mat_mul(vc2m, T, tmp);
    mat_mul(tmp, V, v_T);
    mat_T(g.W, Wt);
    mat_mul(v_T, Wt, v_J);
    float v_t_x = (-fx * rz2) * v_J[2];
    float v_t_y = (-fy * rz2) * v_J[5];
    float v_t_z = (((-fx * rz2) * v_J[0] + (((2.0f * fx) * tx) * rz3) * v_J[2]) - (fy * rz2) * v_J[4]) +
                  (((2.0f * fy) * ty) * rz3) * v_J[5];
    float v_p[3] = {vvx + v_t_x, vvy + v_t_y, vvz + v_t_z};
    float v_mean_world[3], v_Vs[9], v_M_world[9];
    mat_vec(Wt, v_p, v_mean_world);
#pragma unroll
    for (int k = 0; k < 9; ++k) v_Vs[k] = v_V[k] + v_V[3 * (k % 3) + k / 3];
    mat_mul(v_Vs, g.M, v_M_world);
    // _transform_vjp (:536-557)
    float v_mean_out[3], v_M[9];
    if (moved) {
      float Rtt[9], M_local[9], Mlt[9], vMM[9];
      mat_T(g.R_tf, Rtt);
      mat_vec(Rtt, v_mean_world, v_mean_out);
      mat_mul(Rtt, v_M_world, v_M);
      mat_mul(Rtt, g.M, M_local);
      mat_T(M_local, Mlt);
      mat_mul(v_M_world, Mlt, vMM);
      const int64_t m_idx = a.sel_means ? idx : gid;
      const float ml[3] = {a.means[3 * m_idx], a.means[3 * m_idx + 1], a.means[3 * m_idx + 2]};
#pragma unroll
      for (int r = 0; r < 3; ++r) {
#pragma unroll
        for (int c = 0; c < 3; ++c) vtf[4 * r + c] = v_mean_world[r] * ml[c] + vMM[3 * r + c];
        vtf[4 * r + 3] = v_mean_world[r];
      }
    } else {
#pragma unroll
      for (int k = 0; k < 3; ++k) v_mean_out[k] = v_mean_world[k];
#pragma unroll
      for (int k = 0; k < 9; ++k) v_M[k] = v_M_world[k];
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) acc_mean[c] += v_mean_out[c];
    // _scale_vjp (:560-567)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      acc_scale[c] += ((R[c] * v_M[c] + R[3 + c] * v_M[3 + c]) + R[6 + c] * v_M[6 + c]) * gs;
    // _quat_vjp (:570-599), written xyzw
    float vR[9];
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int c = 0; c < 3; ++c) vR[3 * r + c] = v_M[3 * r + c] * s[c];
    const float x = q[0], y = q[1], z = q[2], w = q[3];
    float vq_w = 2.0f * (x * (vR[7] - vR[5]) + y * (vR[2] - vR[6]) + z * (vR[3] - vR[1]));
    float vq_x = 2.0f * (-2.0f * x * (vR[4] + vR[8]) + y * (vR[3] + vR[1]) + z * (vR[6] + vR[2]) +
                         w * (vR[7] - vR[5]));
    float vq_y = 2.0f * (x * (vR[3] + vR[1]) - 2.0f * y * (vR[0] + vR[8]) + z * (vR[7] + vR[5]) +
                         w * (vR[2] - vR[6]));
    float vq_z = 2.0f * (x * (vR[6] + vR[2]) + y * (vR[7] + vR[5]) - 2.0f * z * (vR[0] + vR[4]) +
                         w * (vR[3] - vR[1]));
    acc_quat[0] += vq_x;
    acc_quat[1] += vq_y;
    acc_quat[2] += vq_z;
    acc_quat[3] += vq_w;
    // _view_vjp (:602-606)
    float Jt[9], JtvT[9];
    mat_T(J, Jt);
    mat_mul(Jt, v_T, JtvT);
#pragma unroll
    for (int r = 0; r < 3; ++r) {
#pragma unroll
      for (int c = 0; c < 3; ++c) vv[4 * r + c] = v_p[r] * g.mean[c] + JtvT[3 * r + c];
      vv[4 * r + 3] = v_p[r];
    }
  }
  // per-image viewmat cotangent: warp reduce-scatter, then one atomic per entry per warp
  // (rows image_id*4 + r of the (4B, 4) output; row 3 stays zero)
  {
    const int c = warp_reduce_scatter<12>(vv, lane);
    if (c >= 0 && vv[0] != 0.0f) atomicAdd(&a.v_viewmat[16 * image_id + c], vv[0]);
  }
  // transform cotangent (:461-484): reduce when the block is uniformly on one transform,
  // per-thread atomics otherwise
  if (a.has_transforms) {
    __shared__ int s_tmin, s_tmax;
    if (threadIdx.x == 0) { s_tmin = 0x7fffffff; s_tmax = -0x7fffffff; }
    __syncthreads();
    atomicMin(&s_tmin, tf_id);
    atomicMax(&s_tmax, tf_id);
    __syncthreads();
    const int tmin = s_tmin, tmax = s_tmax;
    if (tmin == tmax && tmin >= 0) {
      const int c = warp_reduce_scatter<12>(vtf, lane);
      if (c >= 0 && vtf[0] != 0.0f)
        atomicAdd(&a.v_transforms[16 * (image_id * a.num_transforms + tmin) + c], vtf[0]);
    } else if (moved) {
      float* out = a.v_transforms + 16 * (image_id * a.num_transforms + tf_id);
#pragma unroll
      for (int k = 0; k < 12; ++k) atomicAdd(&out[k], vtf[k]);
    }
    __syncthreads();  // s_tmin / s_tmax are reset by the next image
  }
  }  // images
  if (gid < a.n) {
    // one row per gaussian (FOLD) or per (image, gaussian); quats in the input's order
    const int64_t row = FOLD ? gid : img0 * a.n + gid;
    a.v_mean3d[3 * row] = acc_mean[0];
    a.v_mean3d[3 * row + 1] = acc_mean[1];
    a.v_mean3d[3 * row + 2] = acc_mean[2];
    a.v_scale[3 * row] = acc_scale[0];
    a.v_scale[3 * row + 1] = acc_scale[1];
    a.v_scale[3 * row + 2] = acc_scale[2];
    float* vq = a.v_quat + 4 * row;
    if (a.quats_wxyz) {
      vq[0] = acc_quat[3];
      vq[1] = acc_quat[0];
      vq[2] = acc_quat[1];
      vq[3] = acc_quat[2];
    } else {
      vq[0] = acc_quat[0];
      vq[1] = acc_quat[1];
      vq[2] = acc_quat[2];
      vq[3] = acc_quat[3];
    }
  }
  (void)warp;
}

}  // namespace

void launch_project_fwd(const ProjectArgs& a, unsigned long long* status, int* ticket,
                        unsigned* err, cudaStream_t stream) {
  const int64_t blocks = project_scan_tiles(a.total);
  if (blocks == 0) return;
  if (a.rho)
    launch_pdl(project_fwd_kernel<true>, static_cast<unsigned>(blocks), kProjThreads, 0, stream, a,
        status, ticket, err);
  else
    launch_pdl(project_fwd_kernel<false>, static_cast<unsigned>(blocks), kProjThreads, 0, stream, a,
        status, ticket, err);
}

int64_t project_scan_tiles(int64_t total) { return (total + kProjTile - 1) / kProjTile; }

void launch_project_bwd(const ProjectBwdArgs& a, cudaStream_t stream) {
  const int64_t blocks_per_image = (a.n + kBwdThreads - 1) / kBwdThreads;
  const int64_t blocks = blocks_per_image * a.B;
  if (blocks == 0) return;
  const unsigned g = static_cast<unsigned>(a.fold_batch ? blocks_per_image : blocks);
  if (a.v_rho) {
    if (a.fold_batch) launch_pdl(project_bwd_kernel<true, true>, g, kBwdThreads, 0, stream, a);
    else launch_pdl(project_bwd_kernel<true, false>, g, kBwdThreads, 0, stream, a);
  } else {
    if (a.fold_batch) launch_pdl(project_bwd_kernel<false, true>, g, kBwdThreads, 0, stream, a);
    else launch_pdl(project_bwd_kernel<false, false>, g, kBwdThreads, 0, stream, a);
  }
}

}  // namespace splax
