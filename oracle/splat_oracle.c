/*
 * CPU restatement of the splax splatting hot path -- TEST INFRASTRUCTURE ONLY.
 * See splat_oracle.h for the scope, the parity pin and the determinism contract.
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fno-fast-math -fopenmp -fPIC -shared.
 */
#include "splat_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BW ORC_BLOCK_WIDTH
/* splax/_intersect.py:19-20 */
static const float GAUSSIAN_EXTEND_SQ = (float)(3.33 * 3.33);
static const float ALPHA_THRESHOLD = (float)(1.0 / 255.0);

static int64_t g_counters[5];

void orc_counters(int64_t out[5]) { memcpy(out, g_counters, sizeof(g_counters)); }

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Float -> int32 truncation with the saturating semantics of the GPU's cvt.rzi.s32.f32
 * (NaN -> 0, out of range -> INT32_MIN / INT32_MAX), which is what Warp's wp.int32(x)
 * lowers to on the device. */
static inline int32_t f2i(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}

static inline int32_t imin(int32_t a, int32_t b) { return a < b ? a : b; }
static inline int32_t imax(int32_t a, int32_t b) { return a > b ? a : b; }
/* wp.min / wp.max on floats: a < b ? a : b (and a > b ? a : b). */
static inline float fmin_w(float a, float b) { return a < b ? a : b; }
static inline float fmax_w(float a, float b) { return a > b ? a : b; }

/* Natural logarithm by the atanh series log(m) = 2 atanh((m-1)/(m+1))
 * (Abramowitz & Stegun 4.1.27) on m in [sqrt(1/2), sqrt(2)), with a Cody-Waite split of ln 2
 * for the exponent. Plain IEEE single-precision operations in a fixed order, so the CUDA
 * kernels evaluate the identical sequence. Accurate to a few ulp; only determinism matters
 * here, since the value feeds the integer tile walk. */
float orc_logf(float x) {
    if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : NAN;
    if (x == INFINITY) return INFINITY;
    int32_t e = 0;
    uint32_t bits = f2u(x);
    if (bits < 0x00800000u) { /* subnormal */
        x = x * 8388608.0f;
        bits = f2u(x);
        e = -23;
    }
    e += (int32_t)(bits >> 23) - 127;
    float m = u2f((bits & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421356f) {
        m = m * 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    float s2 = s * s;
    float p = 0.0909090936f; /* 1/11 */
    p = p * s2 + 0.111111112f; /* 1/9 */
    p = p * s2 + 0.142857149f; /* 1/7 */
    p = p * s2 + 0.200000003f; /* 1/5 */
    p = p * s2 + 0.333333343f; /* 1/3 */
    p = p * s2 + 1.0f;
    float fe = (float)e;
    float lm = (2.0f * s) * p;
    return fe * 0.693145751953125f + (lm + fe * 1.42860677e-06f);
}

/* ------------------------------------------------------------------ small linear algebra */
/* Row-major 3x3. Products accumulate over k in ascending order: (a0*b0 + a1*b1) + a2*b2. */
static void mat_mul(const float A[9], const float B[9], float C[9]) {
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            C[3 * i + j] = (A[3 * i] * B[j] + A[3 * i + 1] * B[3 + j]) + A[3 * i + 2] * B[6 + j];
}
static void mat_T(const float A[9], float C[9]) {
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) C[3 * i + j] = A[3 * j + i];
}
static void mat_vec(const float A[9], const float v[3], float o[3]) {
    for (int i = 0; i < 3; ++i) o[i] = (A[3 * i] * v[0] + A[3 * i + 1] * v[1]) + A[3 * i + 2] * v[2];
}

/* _load_affine, splax/_project/_kernels.py:609-624: rows r0..r0+2 of a (rows, 4) matrix. */
static void load_affine(const float *m, float R[9], float t[3]) {
    for (int i = 0; i < 3; ++i) {
        R[3 * i] = m[4 * i];
        R[3 * i + 1] = m[4 * i + 1];
        R[3 * i + 2] = m[4 * i + 2];
        t[i] = m[4 * i + 3];
    }
}

/* Rotation matrix of a unit xyzw quaternion, the standard form whose derivative
 * _quat_vjp (splax/_project/_kernels.py:570-599) implements. */
static void quat_to_mat(const float q[4], float R[9]) {
    float x = q[0], y = q[1], z = q[2], w = q[3];
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

/* _apply_transform, splax/_project/_kernels.py:627-644. Returns moved. */
static int apply_transform(const float *transforms, int32_t image_id, int32_t num_transforms,
                           int sel_transforms, int32_t tf_id, float mean[3], float R_tf[9]) {
    for (int i = 0; i < 9; ++i) R_tf[i] = (i % 4 == 0) ? 1.0f : 0.0f;
    if (tf_id < 0) return 0;
    int64_t tf_idx = sel_transforms ? (int64_t)image_id * num_transforms + tf_id : tf_id;
    float t[3], o[3];
    load_affine(transforms + tf_idx * 16, R_tf, t);
    mat_vec(R_tf, mean, o);
    for (int i = 0; i < 3; ++i) mean[i] = o[i] + t[i];
    return 1;
}

/* _project_geom, splax/_project/_kernels.py:647-664. */
static void project_geom(const float mean[3], const float q[4], const float scale[3],
                         float glob_scale, const float *viewmat_rows, const float R_tf[9],
                         int moved, float W[9], float p[3], float M[9]) {
    float trans[3], Wm[3];
    load_affine(viewmat_rows, W, trans);
    mat_vec(W, mean, Wm);
    for (int i = 0; i < 3; ++i) p[i] = Wm[i] + trans[i];
    float R[9];
    quat_to_mat(q, R);
    float s[3] = {glob_scale * scale[0], glob_scale * scale[1], glob_scale * scale[2]};
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) M[3 * i + j] = R[3 * i + j] * s[j];
    if (moved) {
        float Mt[9];
        mat_mul(R_tf, M, Mt);
        memcpy(M, Mt, sizeof(Mt));
    }
}

/* ------------------------------------------------------------------ ellipse tile walk */
/* _Ellipse and helpers, splax/_intersect.py:23-183. Component 0 of bbox_* / rect_* is the
 * walk's outer axis. */
typedef struct {
    float A, B, C, disc, t, px, py;
    float bbox_min[2], bbox_max[2], bbox_argmin[2], bbox_argmax[2];
    int32_t rect_min[2], rect_max[2];
    int valid, isY;
} Ellipse;

static void ellipse_init(float A, float B, float C, float t, float px, float py,
                         int32_t tile_width, int32_t tile_height, Ellipse *s) {
    memset(s, 0, sizeof(*s));
    s->A = A; s->B = B; s->C = C; s->t = t; s->px = px; s->py = py;
    float disc = B * B - A * C;
    s->disc = disc;
    float neg_t_over_disc = -t / disc;
    float x_extent = sqrtf(neg_t_over_disc * C);
    float y_extent = sqrtf(neg_t_over_disc * A);
    float bmin[2] = {px - x_extent, py - y_extent};
    float bmax[2] = {px + x_extent, py + y_extent};
    float Bx_over_C = B * x_extent / C;
    float By_over_A = B * y_extent / A;
    float amin[2] = {py + Bx_over_C, px + By_over_A};
    float amax[2] = {py - Bx_over_C, px - By_over_A};
    const float ts = (float)BW;
    int32_t rminx = imax(0, imin(tile_width, f2i(bmin[0] / ts)));
    int32_t rminy = imax(0, imin(tile_height, f2i(bmin[1] / ts)));
    int32_t rmaxx = imax(0, imin(tile_width, f2i(bmax[0] / ts + 1.0f)));
    int32_t rmaxy = imax(0, imin(tile_height, f2i(bmax[1] / ts + 1.0f)));
    int32_t x_span = rmaxx - rminx, y_span = rmaxy - rminy;
    if (y_span * x_span == 0) return;
    int isY = y_span < x_span;
    s->isY = isY;
    if (isY) {
        s->rect_min[0] = rminy; s->rect_min[1] = rminx;
        s->rect_max[0] = rmaxy; s->rect_max[1] = rmaxx;
        s->bbox_min[0] = bmin[1]; s->bbox_min[1] = bmin[0];
        s->bbox_max[0] = bmax[1]; s->bbox_max[1] = bmax[0];
        s->bbox_argmin[0] = amin[1]; s->bbox_argmin[1] = amin[0];
        s->bbox_argmax[0] = amax[1]; s->bbox_argmax[1] = amax[0];
    } else {
        s->rect_min[0] = rminx; s->rect_min[1] = rminy;
        s->rect_max[0] = rmaxx; s->rect_max[1] = rmaxy;
        s->bbox_min[0] = bmin[0]; s->bbox_min[1] = bmin[1];
        s->bbox_max[0] = bmax[0]; s->bbox_max[1] = bmax[1];
        s->bbox_argmin[0] = amin[0]; s->bbox_argmin[1] = amin[1];
        s->bbox_argmax[0] = amax[0]; s->bbox_argmax[1] = amax[1];
    }
    s->valid = 1;
}

/* _ellipse_intersect, splax/_intersect.py:110-133 */
static void ellipse_intersect(const Ellipse *s, float coord, float out[2]) {
    float p_u, p_v, coeff;
    if (s->isY) { p_u = s->py; p_v = s->px; coeff = s->A; }
    else { p_u = s->px; p_v = s->py; coeff = s->C; }
    float h = coord - p_u;
    float sqrt_term = sqrtf(s->disc * h * h + s->t * coeff);
    float bh = (-s->B) * h;
    out[0] = (bh - sqrt_term) / coeff + p_v;
    out[1] = (bh + sqrt_term) / coeff + p_v;
}

/* ellipse_init_span, splax/_intersect.py:136-143 */
static void ellipse_init_span(const Ellipse *s, float out[2]) {
    float min_line0 = (float)s->rect_min[0] * (float)BW;
    if (s->bbox_min[0] <= min_line0) {
        ellipse_intersect(s, min_line0, out);
        return;
    }
    out[0] = s->bbox_max[1];
    out[1] = s->bbox_min[1];
}

/* ellipse_column_tile_range, splax/_intersect.py:146-169. Writes [min_v, max_v) and the
 * rolling intersect pair, which the caller feeds to the next column as I_min. */
static void ellipse_column(int32_t u, const Ellipse *s, float I_min[2], int32_t *min_v,
                           int32_t *max_v) {
    const float block = (float)BW;
    float min_line = (float)u * block;
    float max_line = min_line + block;
    float I_max[2];
    if (max_line <= s->bbox_max[0]) ellipse_intersect(s, max_line, I_max);
    else { I_max[0] = I_min[0]; I_max[1] = I_min[1]; }
    float emin, emax;
    if (min_line <= s->bbox_argmin[1] && s->bbox_argmin[1] < max_line) emin = s->bbox_min[1];
    else emin = fmin_w(I_min[0], I_max[0]);
    if (min_line <= s->bbox_argmax[1] && s->bbox_argmax[1] < max_line) emax = s->bbox_max[1];
    else emax = fmax_w(I_min[1], I_max[1]);
    *min_v = imax(s->rect_min[1], imin(s->rect_max[1], f2i(emin / block)));
    *max_v = imin(s->rect_max[1], imax(s->rect_min[1], f2i(emax / block + 1.0f)));
    I_min[0] = I_max[0];
    I_min[1] = I_max[1];
}

/* ellipse_tile_count, splax/_intersect.py:172-183 */
static int32_t ellipse_tile_count(const Ellipse *s) {
    if (!s->valid) return 0;
    float I[2];
    ellipse_init_span(s, I);
    int32_t count = 0;
    for (int32_t u = s->rect_min[0]; u < s->rect_max[0]; ++u) {
        int32_t mn, mx;
        ellipse_column(u, s, I, &mn, &mx);
        count += mx - mn;
    }
    return count;
}

/* opacity-aware isocontour level, splax/_project/_kernels.py:227 */
static inline float iso_level(float opac) {
    return fmin_w(GAUSSIAN_EXTEND_SQ, 2.0f * orc_logf(opac / ALPHA_THRESHOLD));
}

/* Tile counts of the ellipse walk for given screen-space geometry (radii > 0 rows only):
 * what K5 emits for each gaussian. Test helper for geometry perturbed after projection. */
void orc_tile_counts(const float *xys, const int32_t *radii, const float *conics,
                     const float *map_opac, int64_t opac_rows, int64_t total, int32_t img_h,
                     int32_t img_w, int32_t *counts) {
    int32_t tbx = (img_w + BW - 1) / BW, tby = (img_h + BW - 1) / BW;
    for (int64_t idx = 0; idx < total; ++idx) {
        counts[idx] = 0;
        if (radii[idx] <= 0) continue;
        Ellipse e;
        ellipse_init(conics[3 * idx], conics[3 * idx + 1], conics[3 * idx + 2],
                     iso_level(map_opac[idx % opac_rows]), xys[2 * idx], xys[2 * idx + 1], tbx,
                     tby, &e);
        counts[idx] = ellipse_tile_count(&e);
    }
}

/* ------------------------------------------------------------------ projection forward */
void orc_project(const float *means3d, int64_t means_rows, const float *scales,
                 int64_t scales_rows, const float *quats, int64_t quats_rows,
                 const float *viewmat, int64_t viewmat_rows, const float *opacities,
                 int64_t opac_rows, const float *transforms, int64_t transforms_rows,
                 const int32_t *transform_ids, int32_t n, int32_t num_transforms,
                 int32_t has_transforms, int32_t img_h, int32_t img_w, float fx, float fy,
                 float cx, float cy, float glob_scale, float clip_thresh, int64_t total,
                 float *xys, float *depths, int32_t *radii, float *conics,
                 int32_t *num_tiles_hit, int32_t *cum_tiles_hit, int nthreads) {
    /* batch selectors, splax/_project/_kernels.py:68-75 */
    int sel_means = means_rows > n, sel_scales = scales_rows > n, sel_quats = quats_rows > n;
    int sel_view = viewmat_rows > 4, sel_opac = opac_rows > n;
    int sel_tf = transforms_rows > num_transforms;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 4096)
    for (int64_t idx = 0; idx < total; ++idx) {
        int64_t bid = idx / n, gid = idx % n;
        int64_t m_idx = sel_means ? idx : gid, s_idx = sel_scales ? idx : gid;
        int64_t q_idx = sel_quats ? idx : gid, o_idx = sel_opac ? idx : gid;
        int64_t vb = (sel_view ? bid : 0) * 4;
        xys[2 * idx] = 0.0f; xys[2 * idx + 1] = 0.0f;
        depths[idx] = 0.0f;
        radii[idx] = 0;
        conics[3 * idx] = 0.0f; conics[3 * idx + 1] = 0.0f; conics[3 * idx + 2] = 0.0f;
        num_tiles_hit[idx] = 0;

        float mean[3] = {means3d[3 * m_idx], means3d[3 * m_idx + 1], means3d[3 * m_idx + 2]};
        int32_t tf_id = has_transforms ? transform_ids[gid] : -1;
        float R_tf[9], W[9], p[3], M[9];
        int moved = apply_transform(transforms, (int32_t)bid, num_transforms, sel_tf, tf_id,
                                    mean, R_tf);
        project_geom(mean, quats + 4 * q_idx, scales + 3 * s_idx, glob_scale,
                     viewmat + vb * 4, R_tf, moved, W, p, M);
        if (p[2] <= clip_thresh) continue;
        float Mt[9], V3[9];
        mat_T(M, Mt);
        mat_mul(M, Mt, V3);

        /* EWA projection, splax/_project/_kernels.py:188-212 */
        float tan_fovx = 0.5f * (float)img_w / fx;
        float tan_fovy = 0.5f * (float)img_h / fy;
        float lim_x = 1.3f * tan_fovx, lim_y = 1.3f * tan_fovy;
        float tx = p[0], ty = p[1], tz = p[2];
        tx = tz * fmin_w(lim_x, fmax_w(-lim_x, tx / tz));
        ty = tz * fmin_w(lim_y, fmax_w(-lim_y, ty / tz));
        float rz = 1.0f / tz;
        float rz2 = rz * rz;
        float J[9] = {fx * rz, 0.0f, (-fx * tx) * rz2, 0.0f, fy * rz, (-fy * ty) * rz2,
                      0.0f, 0.0f, 0.0f};
        float T[9], TV[9];
        mat_mul(J, W, T);
        mat_mul(T, V3, TV);
        float c00 = (TV[0] * T[0] + TV[1] * T[1]) + TV[2] * T[2];
        float c01 = (TV[0] * T[3] + TV[1] * T[4]) + TV[2] * T[5];
        float c11 = (TV[3] * T[3] + TV[4] * T[4]) + TV[5] * T[5];
        float cxx = c00 + 0.3f, cxy = c01, cyy = c11 + 0.3f;
        float det = cxx * cyy - cxy * cxy;
        if (det == 0.0f) continue;
        float inv_det = 1.0f / det;
        float conic[3] = {cyy * inv_det, -cxy * inv_det, cxx * inv_det};

        float rw = 1.0f / (p[2] + 1e-6f);
        float center_x = (p[0] * rw) * fx + cx;
        float center_y = (p[1] * rw) * fy + cy;
        int32_t tb_x = (img_w + BW - 1) / BW, tb_y = (img_h + BW - 1) / BW;

        float opac = opacities[o_idx];
        if (opac < ALPHA_THRESHOLD) continue;
        float t = iso_level(opac);
        float ext = sqrtf(t);
        float radius_x = ceilf(ext * sqrtf(cxx));
        float radius_y = ceilf(ext * sqrtf(cyy));
        if (radius_x <= 0.0f && radius_y <= 0.0f) continue;
        if (center_x + radius_x <= 0.0f || center_x - radius_x >= (float)img_w ||
            center_y + radius_y <= 0.0f || center_y - radius_y >= (float)img_h)
            continue;
        Ellipse e;
        ellipse_init(conic[0], conic[1], conic[2], t, center_x, center_y, tb_x, tb_y, &e);
        int32_t count = ellipse_tile_count(&e);
        if (count <= 0) continue;
        num_tiles_hit[idx] = count;
        depths[idx] = p[2];
        radii[idx] = f2i(fmax_w(radius_x, radius_y));
        xys[2 * idx] = center_x; xys[2 * idx + 1] = center_y;
        conics[3 * idx] = conic[0]; conics[3 * idx + 1] = conic[1]; conics[3 * idx + 2] = conic[2];
    }
    /* global inclusive int32 scan, splax/_project/_kernels.py:104-107 (wraps like int32) */
    uint32_t acc = 0;
    for (int64_t i = 0; i < total; ++i) {
        acc += (uint32_t)num_tiles_hit[i];
        cum_tiles_hit[i] = (int32_t)acc;
    }
}

/* ------------------------------------------------------------------ sort and bin */
static int bit_length(int64_t v) {
    int b = 0;
    while (v > 0) { ++b; v >>= 1; }
    return b;
}

int orc_key_bits(int32_t B, int32_t img_h, int32_t img_w, int req, int32_t *tile_n_bits,
                 int32_t *depth_bits) {
    int32_t tbx = (img_w + BW - 1) / BW, tby = (img_h + BW - 1) / BW;
    int64_t num_tiles = (int64_t)tbx * tby;
    int32_t tnb = bit_length(num_tiles - 1), inb = bit_length((int64_t)B - 1);
    int32_t upper = inb + tnb, db = 31 - upper;
    *tile_n_bits = tnb;
    *depth_bits = db;
    int packed = (req == 0) ? (db >= 16) : (req == 32);
    if (!packed && upper > 32) return -1;
    if (packed && db < 1) return -1; /* forced packing without room for any depth bit */
    return packed ? 32 : 64;
}

/* _seed_minmax + _depth_minmax, splax/_rasterize/_sort/_kernels.py:31-73 */
static void depth_minmax(const float *depths, const int32_t *radii, int64_t total, int32_t n,
                         int32_t B, float *mm) {
    for (int32_t b = 0; b < B; ++b) { mm[2 * b] = 1.0e30f; mm[2 * b + 1] = -1.0e30f; }
    for (int64_t idx = 0; idx < total; ++idx) {
        if (radii[idx] <= 0) continue;
        int64_t im = idx / n;
        mm[2 * im] = fmin_w(mm[2 * im], depths[idx]);
        mm[2 * im + 1] = fmax_w(mm[2 * im + 1], depths[idx]);
    }
}

/* _map_intersects_32bit / _64bit, splax/_rasterize/_sort/_kernels.py:76-211 */
static int map_intersects(const float *xys, const float *depths, const int32_t *radii,
                          const float *conics, const float *map_opac, int64_t opac_mod,
                          const int32_t *cum, int32_t n, int32_t B, int32_t img_h,
                          int32_t img_w, int key_bits, int32_t tile_n_bits, int32_t depth_bits,
                          const float *mm, int64_t *keys, int32_t *gids) {
    int32_t tbx = (img_w + BW - 1) / BW, tby = (img_h + BW - 1) / BW;
    int64_t total = (int64_t)B * n;
    int bad = 0;
    for (int64_t idx = 0; idx < total; ++idx) {
        if (radii[idx] <= 0) continue;
        int64_t bid = idx / n;
        int64_t cur = idx > 0 ? cum[idx - 1] : 0;
        int64_t end = cum[idx];
        int64_t enc = 0;
        int32_t depth_q = 0;
        if (key_bits == 32) {
            float dmin = mm[2 * bid];
            float drange = mm[2 * bid + 1] - dmin;
            float maxq = (float)((1 << depth_bits) - 1);
            if (drange > 0.0f) {
                float f = (depths[idx] - dmin) / drange;
                int32_t q = f2i(f * maxq);
                depth_q = imin(imax(q, 0), (1 << depth_bits) - 1);
            }
            enc = bid << (depth_bits + tile_n_bits);
        } else {
            int32_t dbits = (int32_t)f2u(depths[idx]);
            enc = (bid << (32 + tile_n_bits)) | (int64_t)dbits; /* sign-extends, as wp.int64 */
        }
        float opac = map_opac[idx % opac_mod];
        float t = iso_level(opac);
        Ellipse e;
        ellipse_init(conics[3 * idx], conics[3 * idx + 1], conics[3 * idx + 2], t, xys[2 * idx],
                     xys[2 * idx + 1], tbx, tby, &e);
        if (!e.valid) continue;
        float I[2];
        ellipse_init_span(&e, I);
        for (int32_t u = e.rect_min[0]; u < e.rect_max[0]; ++u) {
            int32_t mn, mx;
            ellipse_column(u, &e, I, &mn, &mx);
            for (int32_t v = mn; v < mx; ++v) {
                int64_t tile = e.isY ? (int64_t)u * tbx + v : (int64_t)v * tbx + u;
                if (cur >= end) { bad = 1; break; }
                int64_t key = key_bits == 32 ? (enc | (tile << depth_bits) | depth_q)
                                             : (enc | (tile << 32));
                if (keys) keys[cur] = key;
                gids[cur] = (int32_t)idx;
                ++cur;
            }
        }
        if (cur != end) bad = 1;
    }
    return bad ? -2 : 0;
}

int orc_map_intersects(const float *xys, const float *depths, const int32_t *radii,
                       const float *conics, const float *map_opac, int64_t map_opac_rows,
                       const int32_t *cum, int32_t n, int32_t B, int32_t img_h, int32_t img_w,
                       int key_bits, int64_t *keys, int32_t *gids) {
    int32_t tnb, db;
    int kb = orc_key_bits(B, img_h, img_w, key_bits, &tnb, &db);
    if (kb < 0) return -1;
    float *mm = (float *)malloc(sizeof(float) * 2 * (size_t)(B > 0 ? B : 1));
    depth_minmax(depths, radii, (int64_t)B * n, n, B, mm);
    int rc = map_intersects(xys, depths, radii, conics, map_opac, map_opac_rows, cum, n, B,
                            img_h, img_w, kb, tnb, db, mm, keys, gids);
    free(mm);
    return rc;
}

/* Stable ascending sort of signed 64-bit keys carrying int32 values: an LSD radix sort over
 * 8-bit digits (the semantics of warp.utils.radix_sort_pairs, a stable signed sort). */
static void stable_sort_pairs(int64_t *keys, int32_t *vals, int64_t count) {
    if (count <= 1) return;
    uint64_t *k0 = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)count);
    uint64_t *k1 = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)count);
    int32_t *v1 = (int32_t *)malloc(sizeof(int32_t) * (size_t)count);
    int32_t *v0 = vals;
    uint64_t any = 0;
    for (int64_t i = 0; i < count; ++i) {
        k0[i] = (uint64_t)keys[i] ^ 0x8000000000000000ull; /* signed order */
        any |= k0[i] ^ k0[0];
    }
    for (int pass = 0; pass < 8; ++pass) {
        int shift = pass * 8;
        if (((any >> shift) & 0xffull) == 0) continue; /* every key shares this digit */
        int64_t hist[256];
        memset(hist, 0, sizeof(hist));
        for (int64_t i = 0; i < count; ++i) hist[(k0[i] >> shift) & 0xff]++;
        int64_t run = 0;
        for (int d = 0; d < 256; ++d) { int64_t h = hist[d]; hist[d] = run; run += h; }
        for (int64_t i = 0; i < count; ++i) {
            int64_t dst = hist[(k0[i] >> shift) & 0xff]++;
            k1[dst] = k0[i];
            v1[dst] = v0[i];
        }
        uint64_t *tk = k0; k0 = k1; k1 = tk;
        int32_t *tv = v0; v0 = v1; v1 = tv;
    }
    for (int64_t i = 0; i < count; ++i) keys[i] = (int64_t)(k0[i] ^ 0x8000000000000000ull);
    if (v0 != vals) {
        memcpy(vals, v0, sizeof(int32_t) * (size_t)count);
        v1 = v0;
    }
    free(k0);
    free(k1);
    free(v1);
}

/* _tile_bin_edges_32bit / _64bit, splax/_rasterize/_sort/_kernels.py:214-269 */
static void tile_bin_edges(const int64_t *keys, int64_t count, int key_bits,
                           int32_t num_tiles, int32_t tile_n_bits, int32_t depth_bits,
                           int32_t *bins) {
    int shift = key_bits == 32 ? depth_bits : 32;
    int64_t mask = ((int64_t)1 << tile_n_bits) - 1;
    for (int64_t idx = 0; idx < count; ++idx) {
        int64_t key = keys[idx] >> shift;
        int64_t cur = (key >> tile_n_bits) * num_tiles + (key & mask);
        if (idx == 0) { bins[2 * cur] = 0; continue; }
        if (idx == count - 1) bins[2 * cur + 1] = (int32_t)count;
        int64_t keyp = keys[idx - 1] >> shift;
        int64_t prev = (keyp >> tile_n_bits) * num_tiles + (keyp & mask);
        if (prev != cur) {
            bins[2 * prev + 1] = (int32_t)idx;
            bins[2 * cur] = (int32_t)idx;
        }
    }
    /* As in the reference, index 0 returns before the last-index test, so with exactly one
     * intersection its bin keeps end = 0 and the intersection is never blended. */
}

int orc_sort_and_bin(const float *xys, const float *depths, const int32_t *radii,
                     const float *conics, const float *map_opac, int64_t map_opac_rows,
                     const int32_t *cum, int32_t n, int32_t B, int32_t img_h, int32_t img_w,
                     int key_req, int32_t *gids, int64_t *keys_out, int32_t *bins,
                     int32_t *used_key_bits, int nthreads) {
    (void)nthreads;
    int32_t tnb, db;
    int kb = orc_key_bits(B, img_h, img_w, key_req, &tnb, &db);
    if (used_key_bits) *used_key_bits = kb;
    if (kb < 0) return -1;
    int32_t tbx = (img_w + BW - 1) / BW, tby = (img_h + BW - 1) / BW;
    int32_t num_tiles = tbx * tby;
    int64_t total = (int64_t)B * n;
    memset(bins, 0, sizeof(int32_t) * 2 * (size_t)B * num_tiles);
    int64_t count = total > 0 ? (int64_t)(uint32_t)cum[total - 1] : 0;
    if (count == 0) return 0;
    float *mm = (float *)malloc(sizeof(float) * 2 * (size_t)B);
    depth_minmax(depths, radii, total, n, B, mm);
    int64_t *keys = keys_out ? keys_out : (int64_t *)malloc(sizeof(int64_t) * (size_t)count);
    int rc = map_intersects(xys, depths, radii, conics, map_opac, map_opac_rows, cum, n, B,
                            img_h, img_w, kb, tnb, db, mm, keys, gids);
    free(mm);
    if (rc == 0) {
        stable_sort_pairs(keys, gids, count);
        tile_bin_edges(keys, count, kb, num_tiles, tnb, db, bins);
    }
    if (!keys_out) free(keys);
    return rc;
}

/* ------------------------------------------------------------------ forward blend */
/* True when two correct fp32 evaluation orders may disagree on the decision x < bound. */
static inline int near(float x, float bound, float rel) {
    return fabsf(x - bound) <= rel * fabsf(bound);
}

int orc_rasterize(const float *colors, int64_t color_rows, const float *opacities,
                  int64_t opac_rows, const float *map_opac, int64_t map_opac_rows,
                  const float *background, int64_t bg_rows, const float *xys,
                  const float *depths, const int32_t *radii, const float *conics,
                  const int32_t *cum, int32_t n, int32_t B, int32_t img_h, int32_t img_w,
                  int key_req, float *final_Ts, int32_t *final_idx, float *out_img,
                  float *out_depth, uint8_t *flags, int nthreads) {
    int32_t tbx = (img_w + BW - 1) / BW, tby = (img_h + BW - 1) / BW;
    int32_t num_tiles = tbx * tby;
    int64_t total = (int64_t)B * n;
    int64_t count = total > 0 ? (int64_t)(uint32_t)cum[total - 1] : 0;
    int32_t *gids = (int32_t *)malloc(sizeof(int32_t) * (size_t)(count > 0 ? count : 1));
    int32_t *bins = (int32_t *)malloc(sizeof(int32_t) * 2 * (size_t)B * num_tiles);
    int rc = orc_sort_and_bin(xys, depths, radii, conics, map_opac, map_opac_rows, cum, n, B,
                              img_h, img_w, key_req, gids, NULL, bins, NULL, nthreads);
    if (rc != 0) { free(gids); free(bins); return rc; }
    int sel_bg = bg_rows > 1;
    int64_t evals = 0, contribs = 0;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : evals, contribs)
    for (int64_t tile_g = 0; tile_g < (int64_t)B * num_tiles; ++tile_g) {
        int64_t image_id = tile_g / num_tiles;
        int32_t tile_local = (int32_t)(tile_g % num_tiles);
        int32_t tile_x = tile_local % tbx, tile_y = tile_local / tbx;
        int32_t start = bins[2 * tile_g], end = bins[2 * tile_g + 1];
        const float *bg = background + 3 * (sel_bg ? image_id : 0);
        for (int li = 0; li < BW; ++li) {
            for (int lj = 0; lj < BW; ++lj) {
                int32_t i = tile_y * BW + li, j = tile_x * BW + lj;
                if (i >= img_h || j >= img_w) continue;
                float px = (float)j + 0.5f, py = (float)i + 0.5f;
                float T = 1.0f, pix[3] = {0.0f, 0.0f, 0.0f}, dep = 0.0f;
                int32_t cur_idx = 0;
                uint8_t flag = 0;
                float relT = 0.0f; /* bound on the relative error another fp32 order gives T */
                for (int32_t idx = start; idx < end; ++idx) {
                    int64_t g = gids[idx];
                    float dx = xys[2 * g] - px, dy = xys[2 * g + 1] - py;
                    float a = conics[3 * g], b = conics[3 * g + 1], c = conics[3 * g + 2];
                    float o = opacities[g % opac_rows];
                    float sigma = 0.5f * (a * dx * dx + c * dy * dy) + b * dx * dy;
                    float araw = o * expf(-sigma);
                    float alpha = fmin_w(0.999f, araw);
                    ++evals;
                    float mag = fabsf(0.5f * a * dx * dx) + fabsf(0.5f * c * dy * dy) +
                                fabsf(b * dx * dy);
                    if (sigma != 0.0f && fabsf(sigma) <= 1e-5f * mag && o >= ALPHA_THRESHOLD)
                        flag = 1;
                    /* exp and sigma may each be off by a few ulp, sigma more under cancellation */
                    float rel_a = 1e-5f + 1e-6f * mag;
                    if (near(araw, ALPHA_THRESHOLD, rel_a)) flag = 1;
                    if (sigma < 0.0f || alpha < 1.0f / 255.0f) continue;
                    float next_T = T * (1.0f - alpha);
                    relT = relT + 2.5e-7f + (alpha / (1.0f - alpha)) * rel_a;
                    if (near(next_T, 1e-4f, relT)) flag = 1;
                    if (next_T <= 1e-4f) break;
                    float vis = alpha * T;
                    const float *col = colors + 3 * (g % color_rows);
                    pix[0] = pix[0] + col[0] * vis;
                    pix[1] = pix[1] + col[1] * vis;
                    pix[2] = pix[2] + col[2] * vis;
                    if (out_depth) dep = dep + depths[g] * vis;
                    T = next_T;
                    cur_idx = idx;
                    ++contribs;
                }
                int64_t pi = (image_id * img_h + i) * (int64_t)img_w + j;
                final_Ts[pi] = T;
                final_idx[pi] = cur_idx;
                out_img[3 * pi] = pix[0] + T * bg[0];
                out_img[3 * pi + 1] = pix[1] + T * bg[1];
                out_img[3 * pi + 2] = pix[2] + T * bg[2];
                if (out_depth) out_depth[pi] = dep;
                if (flags) flags[pi] = flag;
            }
        }
    }
    g_counters[0] = count;
    g_counters[1] = evals;
    g_counters[2] = contribs;
    free(gids);
    free(bins);
    return 0;
}

/* ------------------------------------------------------------------ backward blend */
static inline void atomic_addd(double *p, double v) {
#pragma omp atomic
    *p += v;
}

int orc_rasterize_bwd(const float *colors, int64_t color_rows, const float *opacities,
                      int64_t opac_rows, const float *map_opac, int64_t map_opac_rows,
                      const float *background, int64_t bg_rows, const float *xys,
                      const float *depths, const int32_t *radii, const float *conics,
                      const int32_t *cum, const float *final_Ts, const int32_t *final_idx,
                      const float *v_out_img, int64_t vout_rows, const float *v_out_depth,
                      int64_t vdepth_rows, int32_t n, int32_t B_out, int32_t B_geom,
                      int32_t img_h, int32_t img_w, int key_req, float *v_colors,
                      float *v_opacity, float *v_xy, float *v_conic, float *v_depths,
                      int nthreads) {
    int32_t tbx = (img_w + BW - 1) / BW, tby = (img_h + BW - 1) / BW;
    int32_t num_tiles = tbx * tby;
    int64_t total = (int64_t)B_geom * n;
    int64_t count = total > 0 ? (int64_t)(uint32_t)cum[total - 1] : 0;
    int32_t *gids = (int32_t *)malloc(sizeof(int32_t) * (size_t)(count > 0 ? count : 1));
    int32_t *bins = (int32_t *)malloc(sizeof(int32_t) * 2 * (size_t)B_geom * num_tiles);
    int rc = orc_sort_and_bin(xys, depths, radii, conics, map_opac, map_opac_rows, cum, n,
                              B_geom, img_h, img_w, key_req, gids, NULL, bins, NULL, nthreads);
    if (rc != 0) { free(gids); free(bins); return rc; }
    int64_t rows = (int64_t)B_out * n;
    /* per-gaussian accumulator: rgb(3) conic(3) xy(2) opac(1) depth(1) */
    double *acc = (double *)calloc((size_t)rows * 10, sizeof(double));
    int sel_geom = B_geom > 1, sel_bg = bg_rows > 1;
    int64_t evals = 0, contribs = 0;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : evals, contribs)
    for (int64_t tile_g = 0; tile_g < (int64_t)B_out * num_tiles; ++tile_g) {
        int64_t image_id = tile_g / num_tiles;
        int32_t tile_local = (int32_t)(tile_g % num_tiles);
        int64_t geom_image = sel_geom ? image_id : 0;
        int64_t og_base = sel_geom ? 0 : image_id * n;
        int32_t tile_x = tile_local % tbx, tile_y = tile_local / tbx;
        int64_t bin = geom_image * num_tiles + tile_local;
        int32_t start = bins[2 * bin], end = bins[2 * bin + 1];
        if (end <= start) continue;
        const float *bg = background + 3 * (sel_bg ? image_id : 0);
        for (int li = 0; li < BW; ++li) {
            for (int lj = 0; lj < BW; ++lj) {
                int32_t i = tile_y * BW + li, j = tile_x * BW + lj;
                if (i >= img_h || j >= img_w) continue;
                float px = (float)j + 0.5f, py = (float)i + 0.5f;
                int64_t fpi = (geom_image * img_h + i) * (int64_t)img_w + j;
                int32_t bin_final = final_idx[fpi];
                if (bin_final > end - 1) bin_final = end - 1;
                float t_final = final_Ts[fpi];
                float T = t_final;
                int64_t vrow = (image_id * img_h + i) % vout_rows;
                const float *vo = v_out_img + 3 * (vrow * img_w + j);
                float v_outd = 0.0f;
                if (v_out_depth) {
                    int64_t drow = (image_id * img_h + i) % vdepth_rows;
                    v_outd = v_out_depth[drow * img_w + j];
                }
                float buf[3] = {0.0f, 0.0f, 0.0f}, dbuf = 0.0f;
                for (int32_t idx = bin_final; idx >= start; --idx) {
                    int64_t g = gids[idx];
                    float dx = xys[2 * g] - px, dy = xys[2 * g + 1] - py;
                    float a = conics[3 * g], b = conics[3 * g + 1], c = conics[3 * g + 2];
                    float o = opacities[g % opac_rows];
                    float sigma = 0.5f * (a * dx * dx + c * dy * dy) + b * dx * dy;
                    ++evals;
                    if (sigma < 0.0f) continue;
                    float vis = expf(-sigma);
                    float alpha = fmin_w(0.999f, o * vis);
                    if (alpha < 1.0f / 255.0f) continue;
                    ++contribs;
                    const float *col = colors + 3 * (g % color_rows);
                    float dep = v_out_depth ? depths[g] : 0.0f;
                    /* _blend_color_vjp / _blend_depth_vjp, splax/_rasterize/_kernels.py:1212-1302 */
                    float ra = 1.0f / (1.0f - alpha);
                    T = T * ra;
                    float fac = alpha * T;
                    float v_alpha = (col[0] * T - buf[0] * ra) * vo[0];
                    v_alpha += (col[1] * T - buf[1] * ra) * vo[1];
                    v_alpha += (col[2] * T - buf[2] * ra) * vo[2];
                    if (v_out_depth) v_alpha += (dep * T - dbuf * ra) * v_outd;
                    v_alpha += -t_final * ra * bg[0] * vo[0];
                    v_alpha += -t_final * ra * bg[1] * vo[1];
                    v_alpha += -t_final * ra * bg[2] * vo[2];
                    buf[0] = buf[0] + col[0] * fac;
                    buf[1] = buf[1] + col[1] * fac;
                    buf[2] = buf[2] + col[2] * fac;
                    if (v_out_depth) dbuf = dbuf + dep * fac;
                    double *ac = acc + 10 * (og_base + g);
                    atomic_addd(ac + 0, (double)(vo[0] * fac));
                    atomic_addd(ac + 1, (double)(vo[1] * fac));
                    atomic_addd(ac + 2, (double)(vo[2] * fac));
                    if (v_out_depth) atomic_addd(ac + 9, (double)(v_outd * fac));
                    if (o * vis <= 0.999f) {
                        float v_sigma = -o * vis * v_alpha;
                        atomic_addd(ac + 3, (double)(0.5f * v_sigma * dx * dx));
                        atomic_addd(ac + 4, (double)(v_sigma * dx * dy));
                        atomic_addd(ac + 5, (double)(0.5f * v_sigma * dy * dy));
                        atomic_addd(ac + 6, (double)(v_sigma * (a * dx + b * dy)));
                        atomic_addd(ac + 7, (double)(v_sigma * (b * dx + c * dy)));
                        atomic_addd(ac + 8, (double)(vis * v_alpha));
                    }
                }
            }
        }
    }
    for (int64_t r = 0; r < rows; ++r) {
        const double *ac = acc + 10 * r;
        v_colors[3 * r] = (float)ac[0];
        v_colors[3 * r + 1] = (float)ac[1];
        v_colors[3 * r + 2] = (float)ac[2];
        v_conic[3 * r] = (float)ac[3];
        v_conic[3 * r + 1] = (float)ac[4];
        v_conic[3 * r + 2] = (float)ac[5];
        v_xy[2 * r] = (float)ac[6];
        v_xy[2 * r + 1] = (float)ac[7];
        v_opacity[r] = (float)ac[8];
        if (v_depths) v_depths[r] = (float)ac[9];
    }
    g_counters[0] = count;
    g_counters[3] = evals;
    g_counters[4] = contribs;
    free(acc);
    free(gids);
    free(bins);
    return 0;
}

/* ------------------------------------------------------------------ projection backward */
void orc_project_bwd(const float *means3d, int64_t means_rows, const float *scales,
                     int64_t scales_rows, const float *quats, int64_t quats_rows,
                     const float *viewmat, int64_t viewmat_rows, const int32_t *radii,
                     int64_t radii_rows, const float *conics, int64_t conics_rows,
                     const float *v_xy_in, int64_t vxy_rows, const float *v_depth_in,
                     int64_t vdepth_rows, const float *v_conic_in, int64_t vconic_rows,
                     const float *transforms, int64_t transforms_rows,
                     const int32_t *transform_ids, int32_t n, int32_t num_transforms,
                     int32_t has_transforms, float fx, float fy, float glob_scale, int32_t B,
                     float *v_mean3d, float *v_scale, float *v_quat, float *v_viewmat,
                     float *v_transforms, int nthreads) {
    int sel_means = means_rows > n, sel_scales = scales_rows > n, sel_quats = quats_rows > n;
    int sel_view = viewmat_rows > 4, sel_radii = radii_rows > n, sel_conics = conics_rows > n;
    int sel_vxy = vxy_rows > n, sel_vdepth = vdepth_rows > n, sel_vconic = vconic_rows > n;
    int sel_tf = transforms_rows > num_transforms;
    int64_t total = (int64_t)B * n;
    memset(v_mean3d, 0, sizeof(float) * 3 * (size_t)total);
    memset(v_scale, 0, sizeof(float) * 3 * (size_t)total);
    memset(v_quat, 0, sizeof(float) * 4 * (size_t)total);
    double *vview = (double *)calloc((size_t)B * 12, sizeof(double));
    int32_t K = num_transforms > 0 ? num_transforms : 1;
    double *vtf = (double *)calloc((size_t)B * K * 12, sizeof(double));
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 4096)
    for (int64_t idx = 0; idx < total; ++idx) {
        int64_t image_id = idx / n, gid = idx % n;
        int32_t tf_id = has_transforms ? transform_ids[gid] : -1;
        int64_t r_idx = sel_radii ? idx : gid;
        if (radii[r_idx] <= 0) continue;
        int64_t m_idx = sel_means ? idx : gid, s_idx = sel_scales ? idx : gid;
        int64_t q_idx = sel_quats ? idx : gid, c_idx = sel_conics ? idx : gid;
        int64_t vx_idx = sel_vxy ? idx : gid, vd_idx = sel_vdepth ? idx : gid;
        int64_t vc_idx = sel_vconic ? idx : gid;
        int64_t vb = (sel_view ? image_id : 0) * 4;
        const float *ml = means3d + 3 * m_idx;
        float mean_local[3] = {ml[0], ml[1], ml[2]};
        float mean[3] = {ml[0], ml[1], ml[2]};
        float R_tf[9], W[9], p[3], M[9];
        int moved = apply_transform(transforms, (int32_t)image_id, num_transforms, sel_tf, tf_id,
                                    mean, R_tf);
        const float *q = quats + 4 * q_idx;
        const float *sc = scales + 3 * s_idx;
        project_geom(mean, q, sc, glob_scale, viewmat + vb * 4, R_tf, moved, W, p, M);
        float Mt[9], V[9], R[9];
        mat_T(M, Mt);
        mat_mul(M, Mt, V);
        quat_to_mat(q, R);
        float s[3] = {glob_scale * sc[0], glob_scale * sc[1], glob_scale * sc[2]};
        float rz = 1.0f / p[2];
        float rz2 = rz * rz;
        float J[9] = {fx * rz, 0.0f, (-fx * p[0]) * rz2, 0.0f, fy * rz, (-fy * p[1]) * rz2,
                      0.0f, 0.0f, 0.0f};
        float T[9];
        mat_mul(J, W, T);
        const float *conic = conics + 3 * c_idx;
        const float *vcon = v_conic_in + 3 * vc_idx;
        float X[4] = {conic[0], conic[1], conic[1], conic[2]};
        float G[4] = {vcon[0], 0.5f * vcon[1], 0.5f * vcon[1], vcon[2]};
        float XG[4] = {X[0] * G[0] + X[1] * G[2], X[0] * G[1] + X[1] * G[3],
                       X[2] * G[0] + X[3] * G[2], X[2] * G[1] + X[3] * G[3]};
        float S[4] = {XG[0] * X[0] + XG[1] * X[2], XG[0] * X[1] + XG[1] * X[3],
                      XG[2] * X[0] + XG[3] * X[2], XG[2] * X[1] + XG[3] * X[3]};
        float vcov2d[3] = {-S[0], -(S[1] + S[2]), -S[3]};

        /* _proj_vjp, splax/_project/_kernels.py:487-533 */
        const float *vxy = v_xy_in + 2 * vx_idx;
        float vdep = v_depth_in[vd_idx];
        float tx = p[0], ty = p[1], tz = p[2];
        float rz3 = rz2 * rz;
        float rw = 1.0f / (tz + 1e-6f);
        float vpx = fx * vxy[0], vpy = fy * vxy[1];
        float vvx = vpx * rw, vvy = vpy * rw;
        float vvz = (-(vpx * tx + vpy * ty) * rw) * rw;
        vvz = vvz + vdep;
        float vcov[9] = {vcov2d[0], 0.5f * vcov2d[1], 0.0f, 0.5f * vcov2d[1], vcov2d[2], 0.0f,
                         0.0f, 0.0f, 0.0f};
        float Tt[9], tmp[9], v_V[9], v_T[9], Wt[9], v_J[9], vc2[9];
        mat_T(T, Tt);
        mat_mul(Tt, vcov, tmp);
        mat_mul(tmp, T, v_V);
        for (int k = 0; k < 9; ++k) vc2[k] = 2.0f * vcov[k];
        mat_mul(vc2, T, tmp);
        mat_mul(tmp, V, v_T);
        mat_T(W, Wt);
        mat_mul(v_T, Wt, v_J);
        float v_t_x = (-fx * rz2) * v_J[2];
        float v_t_y = (-fy * rz2) * v_J[5];
        float v_t_z = (((-fx * rz2) * v_J[0] + (((2.0f * fx) * tx) * rz3) * v_J[2]) -
                       (fy * rz2) * v_J[4]) +
                      (((2.0f * fy) * ty) * rz3) * v_J[5];
        float v_p[3] = {vvx + v_t_x, vvy + v_t_y, vvz + v_t_z};

        float v_mean_world[3], v_Vs[9], v_M_world[9];
        mat_vec(Wt, v_p, v_mean_world);
        for (int k = 0; k < 9; ++k) v_Vs[k] = v_V[k] + v_V[3 * (k % 3) + k / 3];
        mat_mul(v_Vs, M, v_M_world);

        /* _transform_vjp, splax/_project/_kernels.py:536-557 */
        float v_mean_out[3], v_M[9], v_R_tf[9] = {0}, v_t_tf[3] = {0};
        if (moved) {
            float Rtt[9], M_local[9], Mlt[9], vMM[9];
            mat_T(R_tf, Rtt);
            mat_vec(Rtt, v_mean_world, v_mean_out);
            mat_mul(Rtt, v_M_world, v_M);
            mat_mul(Rtt, M, M_local);
            mat_T(M_local, Mlt);
            mat_mul(v_M_world, Mlt, vMM);
            for (int a = 0; a < 3; ++a)
                for (int b2 = 0; b2 < 3; ++b2)
                    v_R_tf[3 * a + b2] = v_mean_world[a] * mean_local[b2] + vMM[3 * a + b2];
            for (int a = 0; a < 3; ++a) v_t_tf[a] = v_mean_world[a];
        } else {
            memcpy(v_mean_out, v_mean_world, sizeof(v_mean_out));
            memcpy(v_M, v_M_world, sizeof(v_M));
        }
        for (int a = 0; a < 3; ++a) v_mean3d[3 * idx + a] = v_mean_out[a];
        /* _scale_vjp, :560-567 */
        for (int jc = 0; jc < 3; ++jc)
            v_scale[3 * idx + jc] =
                ((R[jc] * v_M[jc] + R[3 + jc] * v_M[3 + jc]) + R[6 + jc] * v_M[6 + jc]) *
                glob_scale;
        /* _quat_vjp, :570-599 */
        float vR[9];
        for (int a = 0; a < 3; ++a)
            for (int b2 = 0; b2 < 3; ++b2) vR[3 * a + b2] = v_M[3 * a + b2] * s[b2];
        float x = q[0], y = q[1], z = q[2], w = q[3];
        float vq_w = 2.0f * (x * (vR[7] - vR[5]) + y * (vR[2] - vR[6]) + z * (vR[3] - vR[1]));
        float vq_x = 2.0f * (-2.0f * x * (vR[4] + vR[8]) + y * (vR[3] + vR[1]) +
                             z * (vR[6] + vR[2]) + w * (vR[7] - vR[5]));
        float vq_y = 2.0f * (x * (vR[3] + vR[1]) - 2.0f * y * (vR[0] + vR[8]) +
                             z * (vR[7] + vR[5]) + w * (vR[2] - vR[6]));
        float vq_z = 2.0f * (x * (vR[6] + vR[2]) + y * (vR[7] + vR[5]) -
                             2.0f * z * (vR[0] + vR[4]) + w * (vR[3] - vR[1]));
        v_quat[4 * idx] = vq_x;
        v_quat[4 * idx + 1] = vq_y;
        v_quat[4 * idx + 2] = vq_z;
        v_quat[4 * idx + 3] = vq_w;
        /* _view_vjp, :602-606 */
        float Jt[9], JtvT[9];
        mat_T(J, Jt);
        mat_mul(Jt, v_T, JtvT);
        double *vv = vview + 12 * image_id;
        for (int a = 0; a < 3; ++a) {
            for (int b2 = 0; b2 < 3; ++b2)
                atomic_addd(vv + 4 * a + b2, (double)(v_p[a] * mean[b2] + JtvT[3 * a + b2]));
            atomic_addd(vv + 4 * a + 3, (double)v_p[a]);
        }
        if (moved) {
            double *vt = vtf + 12 * (image_id * K + tf_id);
            for (int a = 0; a < 3; ++a) {
                for (int b2 = 0; b2 < 3; ++b2) atomic_addd(vt + 4 * a + b2, (double)v_R_tf[3 * a + b2]);
                atomic_addd(vt + 4 * a + 3, (double)v_t_tf[a]);
            }
        }
    }
    for (int32_t b = 0; b < B; ++b) {
        for (int k = 0; k < 16; ++k) v_viewmat[16 * b + k] = k < 12 ? (float)vview[12 * b + k] : 0.0f;
        for (int32_t t = 0; t < num_transforms; ++t)
            for (int k = 0; k < 16; ++k)
                v_transforms[16 * ((int64_t)b * num_transforms + t) + k] =
                    k < 12 ? (float)vtf[12 * ((int64_t)b * K + t) + k] : 0.0f;
    }
    free(vview);
    free(vtf);
}
