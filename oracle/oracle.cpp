// oracle.cpp - CPU restatement of the reference's splat-training hot path.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA path: it
// is loaded by tests/, by __graft_entry__.smoke() and by bench.py's CPU
// baseline leg, and by nothing that ships. It restates, function by
// function, the reference kernels of debsahu/brush (paths below are relative
// to that repository) on the host, with OpenMP over splats / tiles / rows.
//
// Floating point: compiled with -ffp-contract=off so every expression is
// evaluated as written; transcendental functions come from
// include/bsx_fmath.h (the platform-builtin role of the reference's exp/ln).
// Parity pins: the reference's gsplat golden renders (tiny_case, basic_case),
// its raster-oracle known-answer tests, its sort / prefix-sum / tile-offset
// KATs and its loss invariants are checked against this file in tests/.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#include "../include/bsx.h"
#include "../include/bsx_fmath.h"

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };
// Column-major 3x3, c[col][row].
struct M3 { float c[3][3]; };
struct S2 { float c00, c01, c11; };
struct S3 { float c00, c01, c02, c11, c12, c22; };
struct M23 { float c[3][2]; };  // 2x3 column-major: c[col][row]

inline V3 v3(float x, float y, float z) { return V3{x, y, z}; }
inline V3 add(V3 a, V3 b) { return v3(a.x + b.x, a.y + b.y, a.z + b.z); }
inline V3 sub(V3 a, V3 b) { return v3(a.x - b.x, a.y - b.y, a.z - b.z); }
inline V3 scale(V3 a, float s) { return v3(a.x * s, a.y * s, a.z * s); }
inline float dot(V3 a, V3 b) { return (a.x * b.x + a.y * b.y) + a.z * b.z; }
inline bool finite3(V3 a) { return bsx_is_finite(a.x) && bsx_is_finite(a.y) && bsx_is_finite(a.z); }
inline V3 col(const M3& m, int i) { return v3(m.c[i][0], m.c[i][1], m.c[i][2]); }
inline V3 row(const M3& m, int i) { return v3(m.c[0][i], m.c[1][i], m.c[2][i]); }
inline M3 from_cols(V3 a, V3 b, V3 c) {
    M3 m;
    m.c[0][0] = a.x; m.c[0][1] = a.y; m.c[0][2] = a.z;
    m.c[1][0] = b.x; m.c[1][1] = b.y; m.c[1][2] = b.z;
    m.c[2][0] = c.x; m.c[2][1] = c.y; m.c[2][2] = c.z;
    return m;
}
// brush-cube/src/lib.rs:263-268  M * v = (c0*x + c1*y) + c2*z
inline V3 mul_vec3(const M3& m, V3 v) { return add(add(scale(col(m, 0), v.x), scale(col(m, 1), v.y)), scale(col(m, 2), v.z)); }
// brush-cube/src/lib.rs:271-273
inline V3 transpose_mul_vec3(const M3& m, V3 v) { return v3(dot(col(m, 0), v), dot(col(m, 1), v), dot(col(m, 2), v)); }
inline M3 mul_mat3(const M3& m, const M3& n) { return from_cols(mul_vec3(m, col(n, 0)), mul_vec3(m, col(n, 1)), mul_vec3(m, col(n, 2))); }
inline M3 mul_diag(const M3& m, V3 s) { return from_cols(scale(col(m, 0), s.x), scale(col(m, 1), s.y), scale(col(m, 2), s.z)); }

// brush-cube/src/lib.rs:191-216
inline M3 quat_to_mat3(Q4 q) {
    float x2 = q.x * q.x, y2 = q.y * q.y, z2 = q.z * q.z;
    float xy = q.x * q.y, xz = q.x * q.z, yz = q.y * q.z;
    float wx = q.w * q.x, wy = q.w * q.y, wz = q.w * q.z;
    M3 m;
    m.c[0][0] = 1.0f - 2.0f * (y2 + z2); m.c[0][1] = 2.0f * (xy + wz); m.c[0][2] = 2.0f * (xz - wy);
    m.c[1][0] = 2.0f * (xy - wz); m.c[1][1] = 1.0f - 2.0f * (x2 + z2); m.c[1][2] = 2.0f * (yz + wx);
    m.c[2][0] = 2.0f * (xz + wy); m.c[2][1] = 2.0f * (yz - wx); m.c[2][2] = 1.0f - 2.0f * (x2 + y2);
    return m;
}
inline float qdot(Q4 a, Q4 b) { return ((a.w * b.w + a.x * b.x) + a.y * b.y) + a.z * b.z; }
inline Q4 qnormalize(Q4 q) {
    float s = 1.0f / std::sqrt(qdot(q, q));
    return Q4{q.w * s, q.x * s, q.y * s, q.z * s};
}

// brush-cube/src/lib.rs:436-453
inline S2 sym2_inverse(S2 m) {
    float det = m.c00 * m.c11 - m.c01 * m.c01;
    float inv_det = det > 0.0f ? 1.0f / det : 0.0f;
    return S2{m.c11 * inv_det, -m.c01 * inv_det, m.c00 * inv_det};
}
inline float det2_strict(S2 m) { float ad = m.c00 * m.c11; float bc = m.c01 * m.c01; return ad - bc; }
inline bool sym2_finite(S2 m) { return bsx_is_finite(m.c00) && bsx_is_finite(m.c11) && bsx_is_finite(m.c01); }

// brush-cube/src/lib.rs:634-638
inline float calc_sigma(float px, float py, S2 c, float x, float y) {
    float dx = px - x;
    float dy = py - y;
    return 0.5f * (c.c00 * dx * dx + c.c11 * dy * dy) + c.c01 * dx * dy;
}

// e^-sigma of the tile rasterizers (rasterize.rs:120-135): bsx_expf_raster,
// whose domain is [-87, 0]. The kernels evaluate it only for 0 <= sigma <=
// ln(255) + 1 (other pairs are rejected before); here every pair is
// evaluated, so sigma is clamped to the domain first, which changes no
// accepted pair (sigma < 0 and alpha < 1/255 are rejected either way).
inline float raster_gauss(float sigma) { return bsx_expf_raster(-bsx_clamp(sigma, 0.0f, 87.0f)); }

// Which per-pixel arithmetic the rasterizers of this restatement evaluate:
//   0 - the kernels' form: sigma by bsx_raster_sigma (fused products),
//       e^-sigma by bsx_expf_raster, colour sums by fused multiply-add;
//   1 - the reference's expression (rasterize.rs:131-155, rasterize_backwards.rs:325-329):
//       the unfused calc_sigma, e^-sigma correctly rounded from the double
//       exponential, and pix += max(c, 0) * vis.
// Mode 1 measures how far the kernels' arithmetic sits from the reference's
// expression; the parity tests use mode 0.
int g_raster_expr = 0;
inline float raster_sigma_mode(int mode, float c00, float c01, float c11, float dx, float dy) {
    if (mode) return 0.5f * (c00 * dx * dx + c11 * dy * dy) + c01 * dx * dy;
    return bsx_raster_sigma(c00, c01, c11, dx, dy);
}
inline float raster_gauss_mode(int mode, float sigma) {
    return mode ? (float)std::exp(-(double)sigma) : raster_gauss(sigma);
}
inline float raster_accum(int mode, float acc, float c, float v) {
    return mode ? acc + bsx_max(c, 0.0f) * v : bsx_fma(bsx_max(c, 0.0f), v, acc);
}

// kernels/helpers.rs:166-190 (smooth alpha cutoff)
const float kCutMid = 1.0f / 255.0f;
const float kCutBand = 1.0e-3f;
inline float alpha_cutoff_weight(float a) {
    float t = bsx_clamp((a - (kCutMid - 0.5f * kCutBand)) / kCutBand, 0.0f, 1.0f);
    return t * t * (3.0f - 2.0f * t);
}
inline float alpha_cutoff_weight_deriv(float a) {
    float lo = kCutMid - 0.5f * kCutBand, hi = kCutMid + 0.5f * kCutBand;
    bool inside = a > lo && a < hi;
    float t = (a - lo) / kCutBand;
    return inside ? (6.0f * t - 6.0f * t * t) / kCutBand : 0.0f;
}

struct Uni {
    M3 rot; V3 trans;
    float fx, fy, cx, cy;
    float lpx, lpy, lnx, lny;
    V3 cam;
    uint32_t w, h, tbw, tbh;
    float half_max_fov;
    int model;
    float kp[8];
};

Uni uni_from(const bsx_project_uniforms& u) {
    Uni r;
    for (int c = 0; c < 3; ++c)
        for (int k = 0; k < 3; ++k) r.rot.c[c][k] = u.viewmat[c * 3 + k];
    r.trans = v3(u.viewmat[9], u.viewmat[10], u.viewmat[11]);
    r.fx = u.fx; r.fy = u.fy; r.cx = u.cx; r.cy = u.cy;
    r.lpx = u.lim_pos_x; r.lpy = u.lim_pos_y; r.lnx = u.lim_neg_x; r.lny = u.lim_neg_y;
    r.cam = v3(u.camera_pos[0], u.camera_pos[1], u.camera_pos[2]);
    r.w = u.img_w; r.h = u.img_h; r.tbw = u.tile_bw; r.tbh = u.tile_bh;
    r.half_max_fov = u.half_max_render_fov;
    r.model = u.camera_model;
    for (int k = 0; k < 8; ++k) r.kp[k] = u.model_params[k];
    return r;
}

// kernels/camera_model/pinhole.rs:31-56
inline M23 pinhole_jacobian(V3 p, const Uni& u) {
    float inv_z = 1.0f / p.z;
    float dx = u.fx * inv_z;
    float dy = u.fy * inv_z;
    float cxv = bsx_clamp(p.x * inv_z, u.lnx, u.lpx);
    float cyv = bsx_clamp(p.y * inv_z, u.lny, u.lpy);
    M23 j;
    j.c[0][0] = dx; j.c[0][1] = 0.0f;
    j.c[1][0] = 0.0f; j.c[1][1] = dy;
    j.c[2][0] = -dx * cxv; j.c[2][1] = -dy * cyv;
    return j;
}
#include "camera_models.h"

inline cam::Intr intr_of(const Uni& u) { return cam::Intr{u.fx, u.fy, u.cx, u.cy, u.lpx, u.lpy, u.lnx, u.lny, u.kp}; }

// camera_model/mod.rs:48-85: projection and its Jacobian per model
inline void project_point(V3 p, const Uni& u, float* px, float* py) {
    switch (u.model) {
        case 1: cam::kb4_project(p, intr_of(u), px, py); return;
        case 2: cam::rt8_project(p, intr_of(u), px, py); return;
        case 3: cam::tpf_project(p, intr_of(u), px, py); return;
        default: {  // pinhole.rs:24-30
            float inv_z = 1.0f / p.z;
            *px = u.fx * p.x * inv_z + u.cx;
            *py = u.fy * p.y * inv_z + u.cy;
        }
    }
}
inline M23 model_jacobian(V3 p, const Uni& u) {
    switch (u.model) {
        case 1: return cam::kb4_jacobian(p, intr_of(u));
        case 2: return cam::rt8_jacobian(p, intr_of(u));
        case 3: return cam::tpf_jacobian(p, intr_of(u));
        default: return pinhole_jacobian(p, u);
    }
}

// brush-cube/src/lib.rs:333-347  Mat2x3 * v = (c0*x + c1*y) + c2*z
inline void m23_mul_vec3(const M23& m, V3 v, float out[2]) {
    out[0] = (m.c[0][0] * v.x + m.c[1][0] * v.y) + m.c[2][0] * v.z;
    out[1] = (m.c[0][1] * v.x + m.c[1][1] * v.y) + m.c[2][1] * v.z;
}

// kernels/helpers.rs:297-330
S2 calc_cov2d(V3 scl, Q4 quat, V3 mean_c, const Uni& u) {
    M3 ns = mul_diag(mul_mat3(u.rot, quat_to_mat3(quat)), scl);
    M23 j = model_jacobian(mean_c, u);
    M23 v;
    for (int c = 0; c < 3; ++c) m23_mul_vec3(j, col(ns, c), v.c[c]);
    S2 raw;
    raw.c00 = (v.c[0][0] * v.c[0][0] + v.c[1][0] * v.c[1][0]) + v.c[2][0] * v.c[2][0];
    raw.c01 = (v.c[0][0] * v.c[0][1] + v.c[1][0] * v.c[1][1]) + v.c[2][0] * v.c[2][1];
    raw.c11 = (v.c[0][1] * v.c[0][1] + v.c[1][1] * v.c[1][1]) + v.c[2][1] * v.c[2][1];
    const float lim = 1.0e18f;
    float max_abs = bsx_max(bsx_max(std::fabs(raw.c00), std::fabs(raw.c11)), std::fabs(raw.c01));
    float sd = max_abs > lim ? lim / max_abs : 1.0f;
    return S2{raw.c00 * sd, raw.c01 * sd, raw.c11 * sd};
}

// kernels/helpers.rs:335-350
inline S2 compensate_cov2d(S2 c, bool mip, float* filter_comp) {
    float blur = mip ? 0.1f : 0.3f;
    S2 b{c.c00 + blur, c.c01, c.c11 + blur};
    float fc = 1.0f;
    if (mip) {
        float det_raw = bsx_max(det2_strict(c), 0.0f);
        float det_b = det2_strict(b);
        fc = std::sqrt(det_raw / det_b);
    }
    *filter_comp = fc;
    return b;
}

// kernels/helpers.rs:230-241
inline void compute_bbox_extent(S2 conic, float pt, float* ex, float* ey) {
    float det = conic.c00 * conic.c11 - conic.c01 * conic.c01;
    bool degenerate = det <= 0.0f;
    float inv_det = degenerate ? 0.0f : 1.0f / det;
    float x = std::sqrt(2.0f * pt * conic.c11 * inv_det);
    float y = std::sqrt(2.0f * pt * conic.c00 * inv_det);
    *ex = degenerate ? -1.0f : x;
    *ey = degenerate ? -1.0f : y;
}

struct TileBbox { uint32_t min_x, min_y, max_x, max_y; };
// kernels/helpers.rs:262-295
inline TileBbox get_tile_bbox(float cx, float cy, float ex, float ey, uint32_t bw, uint32_t bh) {
    float tw = 16.0f, th = 16.0f;
    float pcx = cx / tw, pcy = cy / th, dx = ex / tw, dy = ey / th;
    float bwf = (float)bw, bhf = (float)bh;
    TileBbox b;
    b.min_x = (uint32_t)bsx_clamp(pcx - dx, 0.0f, bwf);
    b.min_y = (uint32_t)bsx_clamp(pcy - dy, 0.0f, bhf);
    b.max_x = (uint32_t)bsx_clamp(pcx + dx + 1.0f, 0.0f, bwf);
    b.max_y = (uint32_t)bsx_clamp(pcy + dy + 1.0f, 0.0f, bhf);
    return b;
}

// kernels/helpers.rs:385-424 (StopThePop tile test)
inline bool will_primitive_contribute(float rminx, float rminy, float rmaxx, float rmaxy, float mx, float my,
                                      S2 conic, float pt) {
    bool x_left = mx < rminx, x_right = mx > rmaxx;
    bool in_x = !(x_left || x_right);
    bool y_above = my < rminy, y_below = my > rmaxy;
    bool in_y = !(y_above || y_below);
    bool hit = in_x && in_y;
    if (!hit) {
        float corner_x = x_left ? rminx : rmaxx;
        float corner_y = y_above ? rminy : rmaxy;
        float width = rmaxx - rminx;
        float height = rmaxy - rminy;
        float dxf = x_left ? width : -width;
        float dyf = y_above ? height : -height;
        float diff_x = mx - corner_x;
        float diff_y = my - corner_y;
        float tx_raw = (dxf * conic.c00 * diff_x + dxf * conic.c01 * diff_y) / (dxf * conic.c00 * dxf);
        float ty_raw = (dyf * conic.c01 * diff_x + dyf * conic.c11 * diff_y) / (dyf * conic.c11 * dyf);
        float tx = in_y ? 0.0f : bsx_clamp(tx_raw, 0.0f, 1.0f);
        float ty = in_x ? 0.0f : bsx_clamp(ty_raw, 0.0f, 1.0f);
        float max_x = corner_x + tx * dxf;
        float max_y = corner_y + ty * dyf;
        hit = calc_sigma(max_x, max_y, conic, mx, my) <= pt;
    }
    return hit;
}

// kernels/sh.rs:246-336 (Sloan JCGT 2013 basis constants)
V3 sh_coeffs_to_color(const float* c, int degree, V3 v) {
    auto rc = [&](int k) { return v3(c[3 * k], c[3 * k + 1], c[3 * k + 2]); };
    V3 color = scale(rc(0), 0.2820948f);
    if (degree >= 1) {
        const float f0a = 0.4886025f;
        color = add(color, scale(rc(1), -f0a * v.y));
        color = add(color, scale(rc(2), f0a * v.z));
        color = add(color, scale(rc(3), -f0a * v.x));
        if (degree >= 2) {
            float z2 = v.z * v.z;
            float f0b = -1.0925485f * v.z;
            const float f1a = 0.54627424f;
            float fc1 = v.x * v.x - v.y * v.y;
            float fs1 = 2.0f * v.x * v.y;
            float p4 = f1a * fs1, p5 = f0b * v.y, p6 = 0.9461747f * z2 - 0.31539157f, p7 = f0b * v.x, p8 = f1a * fc1;
            color = add(color, scale(rc(4), p4));
            color = add(color, scale(rc(5), p5));
            color = add(color, scale(rc(6), p6));
            color = add(color, scale(rc(7), p7));
            color = add(color, scale(rc(8), p8));
            if (degree >= 3) {
                float f0c = -2.285229f * z2 + 0.4570458f;
                float f1b = 1.4453057f * v.z;
                const float f2a = -0.5900436f;
                float fc2 = v.x * fc1 - v.y * fs1;
                float fs2 = v.x * fs1 + v.y * fc1;
                float p12 = v.z * (1.8658817f * z2 - 1.119529f);
                float p9 = f2a * fs2, p10 = f1b * fs1, p11 = f0c * v.y, p13 = f0c * v.x, p14 = f1b * fc1,
                      p15 = f2a * fc2;
                color = add(color, scale(rc(9), p9));
                color = add(color, scale(rc(10), p10));
                color = add(color, scale(rc(11), p11));
                color = add(color, scale(rc(12), p12));
                color = add(color, scale(rc(13), p13));
                color = add(color, scale(rc(14), p14));
                color = add(color, scale(rc(15), p15));
                if (degree >= 4) {
                    float f0d = v.z * (-4.683326f * z2 + 2.0071396f);
                    float f1c = 3.3116114f * z2 - 0.47308735f;
                    float f2b = -1.7701308f * v.z;
                    const float f3a = 0.62583575f;
                    float fc3 = v.x * fc2 - v.y * fs2;
                    float fs3 = v.x * fs2 + v.y * fc2;
                    float p20 = 1.9843135f * v.z * p12 - 1.0062306f * p6;
                    color = add(color, scale(rc(16), f3a * fs3));
                    color = add(color, scale(rc(17), f2b * fs2));
                    color = add(color, scale(rc(18), f1c * fs1));
                    color = add(color, scale(rc(19), f0d * v.y));
                    color = add(color, scale(rc(20), p20));
                    color = add(color, scale(rc(21), f0d * v.x));
                    color = add(color, scale(rc(22), f1c * fc1));
                    color = add(color, scale(rc(23), f2b * fc2));
                    color = add(color, scale(rc(24), f3a * fc3));
                }
            }
        }
    }
    return color;
}

// kernels/sh.rs:342-470
V3 sh_color_viewdir_vjp(const float* c, int degree, V3 v, V3 vc) {
    auto sd = [&](int k) { return dot(v3(c[3 * k], c[3 * k + 1], c[3 * k + 2]), vc); };
    float gx = 0.0f, gy = 0.0f, gz = 0.0f;
    if (degree >= 1) {
        const float f0a = 0.4886025f;
        float s_n1 = sd(1), s_z0 = sd(2), s_p1 = sd(3);
        gx += -f0a * s_p1;
        gy += -f0a * s_n1;
        gz += f0a * s_z0;
        if (degree >= 2) {
            float z = v.z, x = v.x, y = v.y;
            const float c2 = -1.0925485f, f1a = 0.54627424f;
            float s_n2 = sd(4), s_n1b = sd(5), s_z0b = sd(6), s_p1b = sd(7), s_p2 = sd(8);
            gx += 2.0f * f1a * y * s_n2 + c2 * z * s_p1b + 2.0f * f1a * x * s_p2;
            gy += 2.0f * f1a * x * s_n2 + c2 * z * s_n1b - 2.0f * f1a * y * s_p2;
            gz += c2 * y * s_n1b + 2.0f * 0.9461747f * z * s_z0b + c2 * x * s_p1b;
            if (degree >= 3) {
                float z2 = z * z, x2 = x * x, y2 = y * y;
                const float f2a = -0.5900436f, c1b = 1.4453057f;
                float f1b = c1b * z;
                const float c0c = -2.285229f;
                float f0c = c0c * z2 + 0.4570458f;
                float f0c_dz = 2.0f * c0c * z;
                float s_n3 = sd(9), s_n2c = sd(10), s_n1c = sd(11), s_z0c = sd(12), s_p1c = sd(13), s_p2c = sd(14),
                      s_p3 = sd(15);
                float d12_z = 3.0f * 1.8658817f * z2 - 1.119529f;
                gx += f2a * 6.0f * x * y * s_n3 + 2.0f * f1b * y * s_n2c + f0c * s_p1c + 2.0f * f1b * x * s_p2c +
                      f2a * 3.0f * (x2 - y2) * s_p3;
                gy += f2a * 3.0f * (x2 - y2) * s_n3 + 2.0f * f1b * x * s_n2c + f0c * s_n1c +
                      (-2.0f) * f1b * y * s_p2c + f2a * (-6.0f) * x * y * s_p3;
                gz += 2.0f * c1b * x * y * s_n2c + f0c_dz * y * s_n1c + d12_z * s_z0c + f0c_dz * x * s_p1c +
                      c1b * (x2 - y2) * s_p2c;
                if (degree >= 4) {
                    float fc1 = x2 - y2;
                    float fs1 = 2.0f * x * y;
                    float fc2 = x * fc1 - y * fs1;
                    float fs2 = x * fs1 + y * fc1;
                    float f0d = z * (-4.683326f * z2 + 2.0071396f);
                    float f0d_dz = -14.049978f * z2 + 2.0071396f;
                    float f1c = 3.3116114f * z2 - 0.47308735f;
                    float f1c_dz = 2.0f * 3.3116114f * z;
                    const float f2b_dz_const = -1.7701308f;
                    float f2b = f2b_dz_const * z;
                    const float f3a = 0.62583575f;
                    float p_sh12 = z * (1.8658817f * z2 - 1.119529f);
                    float dp_sh12_dz = 3.0f * 1.8658817f * z2 - 1.119529f;
                    float dp_sh6_dz = 2.0f * 0.9461747f * z;
                    float dp_sh20_dz = 1.9843135f * (p_sh12 + z * dp_sh12_dz) - 1.0062306f * dp_sh6_dz;
                    float s_n4 = sd(16), s_n3d = sd(17), s_n2d = sd(18), s_n1d = sd(19), s_z0d = sd(20),
                          s_p1d = sd(21), s_p2d = sd(22), s_p3d = sd(23), s_p4 = sd(24);
                    gx += f3a * 4.0f * fs2 * s_n4 + f2b * 3.0f * fs1 * s_n3d + f1c * 2.0f * y * s_n2d + f0d * s_p1d +
                          f1c * 2.0f * x * s_p2d + f2b * 3.0f * fc1 * s_p3d + f3a * 4.0f * fc2 * s_p4;
                    gy += f3a * 4.0f * fc2 * s_n4 + f2b * 3.0f * fc1 * s_n3d + f1c * 2.0f * x * s_n2d + f0d * s_n1d +
                          f1c * (-2.0f) * y * s_p2d + f2b * (-3.0f) * fs1 * s_p3d + f3a * (-4.0f) * fs2 * s_p4;
                    gz += f2b_dz_const * fs2 * s_n3d + f1c_dz * fs1 * s_n2d + f0d_dz * y * s_n1d +
                          dp_sh20_dz * s_z0d + f0d_dz * x * s_p1d + f1c_dz * fc1 * s_p2d +
                          f2b_dz_const * fc2 * s_p3d;
                }
            }
        }
    }
    return v3(gx, gy, gz);
}

// kernels/sh.rs:476-555
void sh_coeffs_to_color_vjp(float* out, int degree, V3 v, V3 vc) {
    auto wc = [&](int k, float s) { out[3 * k] = vc.x * s; out[3 * k + 1] = vc.y * s; out[3 * k + 2] = vc.z * s; };
    wc(0, 0.2820948f);
    if (degree >= 1) {
        const float f0a = 0.4886025f;
        wc(1, -f0a * v.y);
        wc(2, f0a * v.z);
        wc(3, -f0a * v.x);
        if (degree >= 2) {
            float z2 = v.z * v.z;
            float f0b = -1.0925485f * v.z;
            const float f1a = 0.54627424f;
            float fc1 = v.x * v.x - v.y * v.y;
            float fs1 = 2.0f * v.x * v.y;
            float p6 = 0.9461747f * z2 - 0.31539157f;
            wc(4, f1a * fs1);
            wc(5, f0b * v.y);
            wc(6, p6);
            wc(7, f0b * v.x);
            wc(8, f1a * fc1);
            if (degree >= 3) {
                float f0c = -2.285229f * z2 + 0.4570458f;
                float f1b = 1.4453057f * v.z;
                const float f2a = -0.5900436f;
                float fc2 = v.x * fc1 - v.y * fs1;
                float fs2 = v.x * fs1 + v.y * fc1;
                float p12 = v.z * (1.8658817f * z2 - 1.119529f);
                wc(9, f2a * fs2);
                wc(10, f1b * fs1);
                wc(11, f0c * v.y);
                wc(12, p12);
                wc(13, f0c * v.x);
                wc(14, f1b * fc1);
                wc(15, f2a * fc2);
                if (degree >= 4) {
                    float f0d = v.z * (-4.683326f * z2 + 2.0071396f);
                    float f1c = 3.3116114f * z2 - 0.47308735f;
                    float f2b = -1.7701308f * v.z;
                    const float f3a = 0.62583575f;
                    float fc3 = v.x * fc2 - v.y * fs2;
                    float fs3 = v.x * fs2 + v.y * fc2;
                    float p20 = 1.9843135f * v.z * p12 + -1.0062306f * p6;
                    wc(16, f3a * fs3);
                    wc(17, f2b * fs2);
                    wc(18, f1c * fs1);
                    wc(19, f0d * v.y);
                    wc(20, p20);
                    wc(21, f0d * v.x);
                    wc(22, f1c * fc1);
                    wc(23, f2b * fc2);
                    wc(24, f3a * fc3);
                }
            }
        }
    }
}

int sh_degree_from_coeffs(uint32_t c) {
    for (int d = 0; d <= 4; ++d)
        if ((uint32_t)((d + 1) * (d + 1)) == c) return d;
    return -1;
}

// Result of one forward render, mirroring render.rs:527-541 plus the
// intermediate arrays the parity tests compare bit-for-bit.
struct Render {
    bsx_project_uniforms uni;
    uint32_t n = 0, num_visible = 0, num_intersections = 0;
    int bwd_info = 0, smooth = 0, mip = 0, degree = 0;
    float bg[3] = {0, 0, 0};
    std::vector<float> projected;        // [N,12]
    std::vector<uint32_t> counts;        // [N]
    std::vector<float> max_radius;       // [N]
    std::vector<uint32_t> depth_order;   // [V] global ids by depth
    std::vector<uint32_t> cum;           // [V]
    std::vector<uint32_t> isect_tile;    // [M] sorted
    std::vector<uint32_t> isect_gid;     // [M] sorted
    std::vector<uint32_t> tile_offsets;  // [T*2]
    std::vector<float> image;            // [H,W,4]
    std::vector<uint32_t> image_packed;  // [H,W]
    std::vector<float> visible;          // [N]
    std::vector<uint32_t> last_useful;   // unused by the reference API; kept for debugging
    int raster_expr = 0;                 // raster arithmetic of this render (g_raster_expr)
};

int g_threads = 0;

}  // namespace

extern "C" {

void orc_set_threads(int n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// camera.rs:49-101,200-254 and render.rs:116-136. glam's Affine3A
// from_rotation_translation(q, p).inverse(): rotation matrix from the
// quaternion, general 3x3 inverse via cross products, translation -(M^-1 p).
// camera.rs:85-198: per-model focal length (f64) and the RT8 clamp-bound undistortion.
static double o_kb4_d(double theta, const float* p) {
    double t2 = theta * theta;
    double t3 = t2 * theta;
    double t5 = t3 * t2;
    double t7 = t5 * t2;
    double t9 = t7 * t2;
    return theta + (double)p[0] * t3 + (double)p[1] * t5 + (double)p[2] * t7 + (double)p[3] * t9;
}
static double o_rt8_radial(double r, const float* p) {
    double r2 = r * r;
    double r4 = r2 * r2;
    double r6 = r4 * r2;
    double num = 1.0 + (double)p[0] * r2 + (double)p[1] * r4 + (double)p[2] * r6;
    double den = 1.0 + (double)p[3] * r2 + (double)p[4] * r4 + (double)p[5] * r6;
    return num / den;
}
static double o_rt8_undistort(double r_d, const float* p) {
    double r = r_d;
    for (int i = 0; i < 30; ++i) {
        double factor = o_rt8_radial(r, p);
        if (std::fabs(factor) < 1e-12) break;
        double r_new = r_d / factor;
        if (std::fabs(r_new - r) < 1e-12) {
            r = r_new;
            break;
        }
        r = r_new;
    }
    return r;
}
static double o_fov_to_focal(double fov, uint32_t pixels, int model, const float* p) {
    double half_fov = fov / 2.0;
    double r_pix = (double)pixels / 2.0;
    double projected;
    switch (model) {
        case 1: case 3: projected = o_kb4_d(half_fov, p); break;
        case 2: { double r = std::tan(half_fov); projected = r * o_rt8_radial(r, p); break; }
        default: projected = std::tan(half_fov);
    }
    return r_pix / projected;
}

int orc_make_project_uniforms(const bsx_camera* cam, uint32_t w, uint32_t h, uint32_t sh_degree,
                              uint32_t total, bsx_project_uniforms* out) {
    if (!cam || !out || cam->camera_model < 0 || cam->camera_model > 3) return 1;
    const int model = cam->camera_model;
    const float* mpar = cam->model_params;
    // glam Mat3A::from_quat (quaternion stored x, y, z, w).
    float qx = cam->rotation[0], qy = cam->rotation[1], qz = cam->rotation[2], qw = cam->rotation[3];
    float x2 = qx + qx, y2 = qy + qy, z2 = qz + qz;
    float xx = qx * x2, xy = qx * y2, xz = qx * z2;
    float yy = qy * y2, yz = qy * z2, zz = qz * z2;
    float wx = qw * x2, wy = qw * y2, wz = qw * z2;
    V3 X = v3(1.0f - (yy + zz), xy + wz, xz - wy);
    V3 Y = v3(xy - wz, 1.0f - (xx + zz), yz + wx);
    V3 Z = v3(xz + wy, yz - wx, 1.0f - (xx + yy));
    auto cross = [](V3 a, V3 b) { return v3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x); };
    V3 t0 = cross(Y, Z), t1 = cross(Z, X), t2 = cross(X, Y);
    float det = dot(Z, t2);
    float inv = 1.0f / det;
    V3 a = scale(t0, inv), b = scale(t1, inv), c = scale(t2, inv);
    // transpose of from_cols(a, b, c): column i = (a[i], b[i], c[i])
    V3 ic0 = v3(a.x, b.x, c.x), ic1 = v3(a.y, b.y, c.y), ic2 = v3(a.z, b.z, c.z);
    V3 p = v3(cam->position[0], cam->position[1], cam->position[2]);
    V3 mp = add(add(scale(ic0, p.x), scale(ic1, p.y)), scale(ic2, p.z));
    V3 tr = v3(-mp.x, -mp.y, -mp.z);
    std::memset(out, 0, sizeof *out);
    float* vm = out->viewmat;
    vm[0] = ic0.x; vm[1] = ic0.y; vm[2] = ic0.z;
    vm[3] = ic1.x; vm[4] = ic1.y; vm[5] = ic1.z;
    vm[6] = ic2.x; vm[7] = ic2.y; vm[8] = ic2.z;
    vm[9] = tr.x; vm[10] = tr.y; vm[11] = tr.z;
    // fov_to_focal (f64) then cast to f32; centre = uv * size (f32)
    double fx = o_fov_to_focal(cam->fov_x, w, model, mpar);
    double fy = o_fov_to_focal(cam->fov_y, h, model, mpar);
    out->fx = (float)fx;
    out->fy = (float)fy;
    out->cx = cam->center_uv[0] * (float)w;
    out->cy = cam->center_uv[1] * (float)h;
    out->camera_pos[0] = p.x; out->camera_pos[1] = p.y; out->camera_pos[2] = p.z;
    float hyp = std::hypot((float)cam->fov_x, (float)cam->fov_y);
    out->half_max_render_fov = bsx_min(hyp * 1.05f, 2.0f * 3.14159265358979323846f - 1e-6f) * 0.5f;
    float wf = (float)w, hf = (float)h;
    if (model == 0 || model == 2) {
        out->lim_pos_x = (1.15f * wf - out->cx) / out->fx;
        out->lim_pos_y = (1.15f * hf - out->cy) / out->fy;
        out->lim_neg_x = (-0.15f * wf - out->cx) / out->fx;
        out->lim_neg_y = (-0.15f * hf - out->cy) / out->fy;
        if (model == 2) {
            float* lims[4] = {&out->lim_pos_x, &out->lim_pos_y, &out->lim_neg_x, &out->lim_neg_y};
            for (float* e : lims) {
                float edge = *e;
                float sign = std::signbit(edge) ? -1.0f : 1.0f;  // f32::signum
                *e = (float)o_rt8_undistort((double)std::fabs(edge), mpar) * sign;
            }
        }
    }
    out->camera_model = model;
    for (int k = 0; k < 8; ++k) out->model_params[k] = mpar[k];
    out->img_w = w; out->img_h = h;
    out->tile_bw = (w + 15) / 16; out->tile_bh = (h + 15) / 16;
    out->sh_degree = sh_degree;
    out->total_splats = total;
    out->num_visible = 0;
    return 0;
}

// Full forward render (render.rs:78-543): project_forward (project_forward.rs:20-144),
// stable depth argsort, count gather + inclusive scan, project_visible
// (project_visible.rs:22-89), map_gaussians (map_gaussians.rs:14-92), stable
// tile argsort, get_tile_offsets (get_tile_offset.rs:10-62), rasterize
// (rasterize.rs:24-200). Ties in depth are broken by global id.
void* orc_render(const bsx_project_uniforms* up, const float* transforms, const float* sh, const float* raw_opac,
                 uint32_t n, uint32_t coeffs, int mip, int pass, const float bg[3]) {
    Render* r = new Render();
    r->uni = *up;
    r->n = n;
    r->mip = mip;
    r->bwd_info = pass != 0;
    r->smooth = pass == 2;
    r->degree = sh_degree_from_coeffs(coeffs);
    r->bg[0] = bg[0]; r->bg[1] = bg[1]; r->bg[2] = bg[2];
    const Uni u = uni_from(*up);
    const uint32_t T = u.tbw * u.tbh;
    r->projected.assign((size_t)n * 12, 0.0f);
    r->counts.assign(n, 0);
    r->max_radius.assign(n, 0.0f);
    std::vector<uint8_t> vis(n, 0);
    std::vector<float> depth(n, 0.0f);

#pragma omp parallel for schedule(dynamic, 1024)
    for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
        const uint32_t g = (uint32_t)gi;
        const float* t = transforms + (size_t)g * 10;
        V3 mean = v3(t[0], t[1], t[2]);
        V3 mean_c = add(mul_vec3(u.rot, mean), u.trans);
        if (!(finite3(mean_c) && mean_c.z <= 1.0e10f)) continue;
        if (u.model == 0) {
            if (mean_c.z < 0.01f) continue;
        } else {  // project_forward.rs:49-64
            float rr = std::sqrt(mean_c.x * mean_c.x + mean_c.y * mean_c.y);
            float theta = bsx_atan2f(rr, mean_c.z);
            if (theta > u.half_max_fov) continue;
        }
        V3 scl = v3(bsx_expf(t[7]), bsx_expf(t[8]), bsx_expf(t[9]));
        if (!finite3(scl)) continue;
        Q4 qu{t[3], t[4], t[5], t[6]};
        float qn = qdot(qu, qu);
        if (!(qn >= 1.0e-6f && bsx_is_finite(qn))) continue;
        float ro = raw_opac[g];
        if (!bsx_is_finite(ro)) continue;
        Q4 q = qnormalize(qu);
        S2 raw = calc_cov2d(scl, q, mean_c, u);
        float fc;
        S2 cov = compensate_cov2d(raw, mip != 0, &fc);
        float opac = bsx_sigmoid(ro) * fc;
        if (!sym2_finite(cov)) continue;
        float m2x, m2y;
        project_point(mean_c, u, &m2x, &m2y);
        if (!(opac >= 1.0f / 255.0f)) continue;
        float pt = bsx_logf(opac * 255.0f);
        S2 conic = sym2_inverse(cov);
        float ex, ey;
        compute_bbox_extent(conic, pt, &ex, &ey);
        if (!(ex >= 0.0f && ey >= 0.0f)) continue;
        float wf = (float)u.w, hf = (float)u.h;
        bool on_screen = m2x + ex > 0.0f && m2x - ex < wf && m2y + ey > 0.0f && m2y - ey < hf;
        if (!on_screen) continue;
        TileBbox bb = get_tile_bbox(m2x, m2y, ex, ey, u.tbw, u.tbh);
        uint32_t hits = 0;
        for (uint32_t ty = bb.min_y; ty < bb.max_y; ++ty)
            for (uint32_t tx = bb.min_x; tx < bb.max_x; ++tx) {
                float rx = (float)(tx * 16u), ry = (float)(ty * 16u);
                if (will_primitive_contribute(rx, ry, rx + 16.0f, ry + 16.0f, m2x, m2y, conic, pt)) ++hits;
            }
        r->counts[g] = hits;
        r->max_radius[g] = bsx_max(ex / wf, ey / hf);
        vis[g] = 1;
        depth[g] = mean_c.z;
        // project_visible: colour from SH at the normalised view direction.
        V3 dv = sub(mean, u.cam);
        V3 vdir = scale(dv, 1.0f / std::sqrt(dot(dv, dv)));
        V3 col = sh_coeffs_to_color(sh + (size_t)g * coeffs * 3, r->degree, vdir);
        float cr = col.x + 0.5f, cg = col.y + 0.5f, cb = col.z + 0.5f;
        cr = bsx_clamp(bsx_is_finite(cr) ? cr : 0.0f, -100.0f, 100.0f);
        cg = bsx_clamp(bsx_is_finite(cg) ? cg : 0.0f, -100.0f, 100.0f);
        cb = bsx_clamp(bsx_is_finite(cb) ? cb : 0.0f, -100.0f, 100.0f);
        float* p = &r->projected[(size_t)g * 12];
        p[0] = m2x; p[1] = m2y; p[2] = conic.c00; p[3] = conic.c01; p[4] = conic.c11;
        p[5] = opac; p[6] = cr; p[7] = cg; p[8] = cb; p[9] = mean_c.z; p[10] = pt; p[11] = 0.0f;
    }

    // Visible list in global-id order, stable-sorted by depth bits (depth > 0).
    std::vector<uint32_t> vlist;
    vlist.reserve(n);
    for (uint32_t g = 0; g < n; ++g)
        if (vis[g]) vlist.push_back(g);
    std::stable_sort(vlist.begin(), vlist.end(), [&](uint32_t a, uint32_t b) {
        return bsx_f32_to_bits(depth[a]) < bsx_f32_to_bits(depth[b]);
    });
    r->depth_order = vlist;
    const uint32_t V = (uint32_t)vlist.size();
    r->num_visible = V;
    r->uni.num_visible = V;
    r->cum.resize(V);
    uint32_t acc = 0;
    for (uint32_t i = 0; i < V; ++i) {
        acc += r->counts[vlist[i]];
        r->cum[i] = acc;
    }
    const uint32_t M = acc;
    r->num_intersections = M;
    std::vector<uint32_t> tile_id(M), gid(M);
#pragma omp parallel for schedule(dynamic, 256)
    for (int64_t ii = 0; ii < (int64_t)V; ++ii) {
        uint32_t i = (uint32_t)ii;
        uint32_t g = vlist[i];
        const float* p = &r->projected[(size_t)g * 12];
        S2 conic{p[2], p[3], p[4]};
        float pt = bsx_logf(p[5] * 255.0f);
        float ex, ey;
        compute_bbox_extent(conic, pt, &ex, &ey);
        TileBbox bb = get_tile_bbox(p[0], p[1], ex, ey, u.tbw, u.tbh);
        uint32_t base = i == 0 ? 0 : r->cum[i - 1];
        uint32_t budget = r->cum[i] - base;
        uint32_t hit = 0;
        for (uint32_t ty = bb.min_y; ty < bb.max_y && hit < budget; ++ty)
            for (uint32_t tx = bb.min_x; tx < bb.max_x && hit < budget; ++tx) {
                float rx = (float)(tx * 16u), ry = (float)(ty * 16u);
                if (will_primitive_contribute(rx, ry, rx + 16.0f, ry + 16.0f, p[0], p[1], conic, pt)) {
                    tile_id[base + hit] = tx + ty * u.tbw;
                    gid[base + hit] = g;
                    ++hit;
                }
            }
        for (uint32_t k = hit; k < budget; ++k) {
            tile_id[base + k] = T;
            gid[base + k] = g;
        }
    }
    // Stable sort by tile id (bits = 32 - lzcnt(T) covers the sentinel T).
    std::vector<uint32_t> order(M);
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return tile_id[a] < tile_id[b]; });
    r->isect_tile.resize(M);
    r->isect_gid.resize(M);
    for (uint32_t k = 0; k < M; ++k) {
        r->isect_tile[k] = tile_id[order[k]];
        r->isect_gid[k] = gid[order[k]];
    }
    r->tile_offsets.assign((size_t)T * 2, 0);
    for (uint32_t k = 0; k < M; ++k) {
        uint32_t tid = r->isect_tile[k];
        if (k == 0) {
            if (tid < T) r->tile_offsets[tid * 2] = 0;
        } else {
            uint32_t prev = r->isect_tile[k - 1];
            if (tid != prev) {
                if (prev < T) r->tile_offsets[prev * 2 + 1] = k;
                if (tid < T) r->tile_offsets[tid * 2] = k;
            }
        }
        if (k == M - 1 && tid < T) r->tile_offsets[tid * 2 + 1] = k + 1;
    }

    // Rasterize (rasterize.rs:118-291), one tile at a time.
    const uint32_t W = u.w, H = u.h;
    const int mode = g_raster_expr;
    r->raster_expr = mode;
    if (r->bwd_info) {
        r->image.assign((size_t)W * H * 4, 0.0f);
        r->visible.assign(n, 0.0f);
    } else {
        r->image_packed.assign((size_t)W * H, 0);
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t ti = 0; ti < (int64_t)T; ++ti) {
        uint32_t tile = (uint32_t)ti;
        uint32_t lo = r->tile_offsets[tile * 2], hi = r->tile_offsets[tile * 2 + 1];
        uint32_t tx = tile % u.tbw, ty = tile / u.tbw;
        uint32_t max_useful = lo;
        for (uint32_t py = ty * 16; py < ty * 16 + 16; ++py)
            for (uint32_t px = tx * 16; px < tx * 16 + 16; ++px) {
                bool inside = px < W && py < H;
                if (!inside) continue;
                float pcx = (float)px + 0.5f, pcy = (float)py + 0.5f;
                float T_acc = 1.0f, pr = 0.0f, pg = 0.0f, pb = 0.0f;
                uint32_t last = lo;
                for (uint32_t k = lo; k < hi; ++k) {
                    uint32_t g = r->isect_gid[k];
                    const float* p = &r->projected[(size_t)g * 12];
                    float sigma = raster_sigma_mode(mode, p[2], p[3], p[4], pcx - p[0], pcy - p[1]);
                    float alpha = bsx_min(0.999f, p[5] * raster_gauss_mode(mode, sigma));
                    float w_cut = r->smooth ? alpha_cutoff_weight(alpha) : (alpha >= kCutMid ? 1.0f : 0.0f);
                    if (sigma >= 0.0f && w_cut > 0.0f) {
                        float ae = alpha * w_cut;
                        float next_t = T_acc * (1.0f - ae);
                        if (next_t <= 1.0e-4f) break;
                        if (r->bwd_info) {
#pragma omp atomic write
                            r->visible[g] = 1.0f;
                        }
                        float v = ae * T_acc;
                        pr = raster_accum(mode, pr, p[6], v);
                        pg = raster_accum(mode, pg, p[7], v);
                        pb = raster_accum(mode, pb, p[8], v);
                        T_acc = next_t;
                        last = k + 1;
                    }
                }
                max_useful = std::max(max_useful, last);
                float fr = pr + T_acc * r->bg[0], fg = pg + T_acc * r->bg[1], fb = pb + T_acc * r->bg[2];
                float fa = 1.0f - T_acc;
                size_t pid = (size_t)py * W + px;
                if (r->bwd_info) {
                    float* o = &r->image[pid * 4];
                    o[0] = fr; o[1] = fg; o[2] = fb; o[3] = fa;
                } else {
                    uint32_t cr = (uint32_t)bsx_clamp(fr * 255.0f, 0.0f, 255.0f);
                    uint32_t cg = (uint32_t)bsx_clamp(fg * 255.0f, 0.0f, 255.0f);
                    uint32_t cb = (uint32_t)bsx_clamp(fb * 255.0f, 0.0f, 255.0f);
                    uint32_t ca = (uint32_t)bsx_clamp(fa * 255.0f, 0.0f, 255.0f);
                    r->image_packed[pid] = cr | (cg << 8) | (cb << 16) | (ca << 24);
                }
            }
        if (r->bwd_info) r->tile_offsets[tile * 2 + 1] = max_useful;
    }
    return r;
}

void orc_render_free(void* h) { delete (Render*)h; }

// Sizes: [num_visible, num_intersections, tile_bw, tile_bh]
void orc_render_sizes(void* h, uint32_t out[4]) {
    Render* r = (Render*)h;
    out[0] = r->num_visible;
    out[1] = r->num_intersections;
    out[2] = r->uni.tile_bw;
    out[3] = r->uni.tile_bh;
}

// Copy one named array out of a render result. Returns element count copied.
size_t orc_render_get(void* h, int which, void* dst) {
    Render* r = (Render*)h;
    auto cp = [&](const void* src, size_t count, size_t elem) {
        if (dst && count) std::memcpy(dst, src, count * elem);
        return count;
    };
    switch (which) {
        case 0: return cp(r->projected.data(), r->projected.size(), 4);
        case 1: return cp(r->counts.data(), r->counts.size(), 4);
        case 2: return cp(r->max_radius.data(), r->max_radius.size(), 4);
        case 3: return cp(r->depth_order.data(), r->depth_order.size(), 4);
        case 4: return cp(r->cum.data(), r->cum.size(), 4);
        case 5: return cp(r->isect_tile.data(), r->isect_tile.size(), 4);
        case 6: return cp(r->isect_gid.data(), r->isect_gid.size(), 4);
        case 7: return cp(r->tile_offsets.data(), r->tile_offsets.size(), 4);
        case 8: return cp(r->image.data(), r->image.size(), 4);
        case 9: return cp(r->image_packed.data(), r->image_packed.size(), 4);
        case 10: return cp(r->visible.data(), r->visible.size(), 4);
        case 11: return cp(&r->uni, 1, sizeof(bsx_project_uniforms));
        default: return 0;
    }
}

// Raster backward (rasterize_backwards.rs:79-443). Per tile, batches of 32
// splats in front-to-back order; every splat visits the tile's pixels in
// row-major order against the running per-pixel state, exactly the order the
// reference's diagonal schedule realises. Per-(tile,batch) partial sums are
// added into v_combined [N,11] (global-id rows).
void orc_rasterize_bwd(void* h, const float* v_output, int compute_refine, float* v_combined) {
    Render* r = (Render*)h;
    const Uni u = uni_from(r->uni);
    const uint32_t W = u.w, H = u.h, T = u.tbw * u.tbh;
    std::memset(v_combined, 0, sizeof(float) * (size_t)r->n * 11);
    const float bgr = r->bg[0], bgg = r->bg[1], bgb = r->bg[2];
    const int mode = r->raster_expr;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t ti = 0; ti < (int64_t)T; ++ti) {
        uint32_t tile = (uint32_t)ti;
        uint32_t lo = r->tile_offsets[tile * 2], hi = r->tile_offsets[tile * 2 + 1];
        if (hi <= lo) continue;
        uint32_t ox = (tile % u.tbw) * 16, oy = (tile / u.tbw) * 16;
        float st[256][4];
        for (uint32_t p = 0; p < 256; ++p) {
            uint32_t px = ox + p % 16, py = oy + p / 16;
            if (px < W && py < H) {
                const float* o = &r->image[((size_t)py * W + px) * 4];
                float tf = 1.0f - o[3];
                st[p][0] = o[0] - tf * bgr;
                st[p][1] = o[1] - tf * bgg;
                st[p][2] = o[2] - tf * bgb;
                st[p][3] = 1.0f;
            } else {
                st[p][0] = st[p][1] = st[p][2] = st[p][3] = 0.0f;
            }
        }
        for (uint32_t k = lo; k < hi; ++k) {
            uint32_t g = r->isect_gid[k];
            const float* s = &r->projected[(size_t)g * 12];
            float sx = s[0], sy = s[1], c00 = s[2], c01 = s[3], c11 = s[4], ca = s[5];
            float crr = s[6], cgg = s[7], cbb = s[8];
            float clr = bsx_max(crr, 0.0f), clg = bsx_max(cgg, 0.0f), clb = bsx_max(cbb, 0.0f);
            float gr[11] = {0};
            for (uint32_t p = 0; p < 256; ++p) {
                float sw = st[p][3];
                if (!(sw > 1.0e-4f)) continue;
                uint32_t px = ox + p % 16, py = oy + p / 16;
                float pcx = (float)px + 0.5f, pcy = (float)py + 0.5f;
                float dx = sx - pcx, dy = sy - pcy;
                float sigma = raster_sigma_mode(mode, c00, c01, c11, dx, dy);
                float gauss = raster_gauss_mode(mode, sigma);
                float alpha = bsx_min(0.999f, ca * gauss);
                float w_cut = r->smooth ? alpha_cutoff_weight(alpha) : (alpha >= kCutMid ? 1.0f : 0.0f);
                if (!(sigma >= 0.0f && w_cut > 0.0f)) continue;
                float ae = alpha * w_cut;
                float next_t = sw * (1.0f - ae);
                if (next_t <= 1.0e-4f) {
                    st[p][3] = 0.0f;
                    continue;
                }
                float vis = ae * sw;
                size_t pid = (size_t)py * W + px;
                const float* vo = &v_output[pid * 4];
                float vox = vo[0], voy = vo[1], voz = vo[2], va = vo[3];
                float fa = r->image[pid * 4 + 3];
                float tf = 1.0f - fa;
                float vow = (va - (bgr * vox + bgg * voy + bgb * voz)) * tf;
                gr[5] += crr >= 0.0f ? vis * vox : 0.0f;
                gr[6] += cgg >= 0.0f ? vis * voy : 0.0f;
                gr[7] += cbb >= 0.0f ? vis * voz : 0.0f;
                float ra = 1.0f / (1.0f - ae);
                float dot_rgb = ((sw * clr - st[p][0]) * vox + (sw * clg - st[p][1]) * voy +
                                 (sw * clb - st[p][2]) * voz) * ra;
                float nrx = st[p][0] - vis * clr, nry = st[p][1] - vis * clg, nrz = st[p][2] - vis * clb;
                float vae = dot_rgb + vow * ra;
                float dw = r->smooth ? alpha_cutoff_weight_deriv(alpha) : 0.0f * alpha;
                float valpha = vae * (w_cut + alpha * dw);
                float vsig = -alpha * valpha;
                float vxx = vsig * (c00 * dx + c01 * dy);
                float vxy = vsig * (c01 * dx + c11 * dy);
                if (ca * gauss <= 0.999f) {
                    gr[2] += 0.5f * vsig * dx * dx;
                    gr[3] += vsig * dx * dy;
                    gr[4] += 0.5f * vsig * dy * dy;
                    gr[0] += vxx;
                    gr[1] += vxy;
                    gr[8] += valpha * gauss;
                    if (compute_refine) {
                        float wf = (float)W, hf = (float)H;
                        float len = std::sqrt(vxx * wf * vxx * wf + vxy * hf * vxy * hf);
                        gr[9] += len / bsx_max(fa, 1.0e-5f);
                    }
                }
                st[p][0] = nrx; st[p][1] = nry; st[p][2] = nrz; st[p][3] = next_t;
            }
            // one batch of 32 ends at (k - lo) % 32 == 31 or at hi; the partial
            // sums per splat are per batch, which for one splat is just gr.
            float* dst = &v_combined[(size_t)g * 11];
            for (int l = 0; l < 11; ++l) {
                if (l == 9 && !compute_refine) continue;
                if (l == 10) continue;
#pragma omp atomic
                dst[l] += gr[l];
            }
        }
    }
}

// Project backward (project_backwards.rs:101-263), dense outputs.
void orc_project_bwd(const bsx_project_uniforms* up, const float* transforms, const float* sh, const float* raw_opac,
                     uint32_t n, uint32_t coeffs, int mip, const float* v_combined, float* v_transforms,
                     float* v_sh, float* v_opac, float* v_refine) {
    const Uni u = uni_from(*up);
    const int degree = sh_degree_from_coeffs(coeffs);
#pragma omp parallel for schedule(static)
    for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
        const uint32_t g = (uint32_t)gi;
        float* vt = v_transforms + (size_t)g * 10;
        float* vs = v_sh + (size_t)g * coeffs * 3;
        for (int k = 0; k < 10; ++k) vt[k] = 0.0f;
        for (uint32_t k = 0; k < coeffs * 3; ++k) vs[k] = 0.0f;
        v_opac[g] = 0.0f;
        v_refine[g] = 0.0f;
        const float* rg = v_combined + (size_t)g * 11;
        bool any = false;
        for (int k = 0; k < 11; ++k) any = any || rg[k] != 0.0f;
        if (!any) continue;
        float vmx = rg[0], vmy = rg[1], vcx = rg[2], vcy = rg[3], vcz = rg[4];
        V3 vcol = v3(rg[5], rg[6], rg[7]);
        float valpha = rg[8], vref = rg[9], vdep = rg[10];
        const float* t = transforms + (size_t)g * 10;
        V3 mean = v3(t[0], t[1], t[2]);
        V3 scl = v3(bsx_expf(t[7]), bsx_expf(t[8]), bsx_expf(t[9]));
        Q4 qu{t[3], t[4], t[5], t[6]};
        Q4 q = qnormalize(qu);
        V3 uw = sub(mean, u.cam);
        float ulen = std::sqrt(dot(uw, uw));
        V3 vdir = scale(uw, 1.0f / ulen);
        const float* shc = sh + (size_t)g * coeffs * 3;
        sh_coeffs_to_color_vjp(vs, degree, vdir, vcol);
        V3 vv = sh_color_viewdir_vjp(shc, degree, vdir, vcol);
        float vdv = dot(vdir, vv);
        V3 v_mean_sh = scale(sub(vv, scale(vdir, vdv)), 1.0f / ulen);
        V3 mean_c = add(mul_vec3(u.rot, mean), u.trans);
        M3 R = quat_to_mat3(q);
        M3 Mm = mul_diag(R, scl);
        S2 raw = calc_cov2d(scl, q, mean_c, u);
        float fc;
        S2 cov = compensate_cov2d(raw, mip != 0, &fc);
        float os = bsx_sigmoid(raw_opac[g]);
        v_opac[g] = fc * valpha * os * (1.0f - os);
        float rc = bsx_is_finite(vref) ? vref : 0.0f;
        v_refine[g] = bsx_clamp(rc, 0.0f, 1.0e32f);
        S2 ci = sym2_inverse(cov);
        S2 vi{vcx, vcy * 0.5f, vcz};
        // inverse2x2_vjp (project_backwards.rs:87-99)
        float t00 = -ci.c00 * vi.c00 + -ci.c01 * vi.c01;
        float t01 = -ci.c01 * vi.c00 + -ci.c11 * vi.c01;
        float t10 = -ci.c00 * vi.c01 + -ci.c01 * vi.c11;
        float t11 = -ci.c01 * vi.c01 + -ci.c11 * vi.c11;
        S2 vcov{t00 * ci.c00 + t10 * ci.c01, t01 * ci.c00 + t11 * ci.c01, t01 * ci.c01 + t11 * ci.c11};
        // covar = M M^T (brush-cube/src/lib.rs:306-318)
        V3 r0 = row(Mm, 0), r1 = row(Mm, 1), r2 = row(Mm, 2);
        S3 covar{dot(r0, r0), dot(r0, r1), dot(r0, r2), dot(r1, r1), dot(r1, r2), dot(r2, r2)};
        // congruence R_view covar R_view^T (lib.rs:515-527)
        auto s3mul = [](const S3& s, V3 v) {
            V3 a = v3(s.c00, s.c01, s.c02), b = v3(s.c01, s.c11, s.c12), c = v3(s.c02, s.c12, s.c22);
            return add(add(scale(a, v.x), scale(b, v.y)), scale(c, v.z));
        };
        V3 vr0 = row(u.rot, 0), vr1 = row(u.rot, 1), vr2 = row(u.rot, 2);
        V3 sr0 = s3mul(covar, vr0), sr1 = s3mul(covar, vr1), sr2 = s3mul(covar, vr2);
        S3 cov_c{dot(vr0, sr0), dot(vr0, sr1), dot(vr0, sr2), dot(vr1, sr1), dot(vr1, sr2), dot(vr2, sr2)};
        M23 J = model_jacobian(mean_c, u);
        // calculate_projection_vjp_pinhole (pinhole.rs:58-123); other models below
        float mx = mean_c.x, my = mean_c.y, mz = mean_c.z;
        float inv_z = 1.0f / mz;
        float mxr = mx * inv_z, myr = my * inv_z;
        float mxc = bsx_clamp(mxr, u.lnx, u.lpx), myc = bsx_clamp(myr, u.lny, u.lpy);
        bool in_x = mxr <= u.lpx && mxr >= u.lnx;
        bool in_y = myr <= u.lpy && myr >= u.lny;
        float iz2 = inv_z * inv_z, iz3 = iz2 * inv_z;
        float v_mx = u.fx * inv_z * vmx;
        float v_my = u.fy * inv_z * vmy;
        float v_mz = -(u.fx * mx * vmx + u.fy * my * vmy) * iz2;
        // tmp = v_cov2d * J: Sym2::mul_mat2x3 -> columns sym * J.col
        float tmp[3][2];
        for (int c = 0; c < 3; ++c) {
            float jx = J.c[c][0], jy = J.c[c][1];
            tmp[c][0] = vcov.c00 * jx + vcov.c01 * jy;
            tmp[c][1] = vcov.c01 * jx + vcov.c11 * jy;
        }
        V3 tr0 = v3(tmp[0][0], tmp[1][0], tmp[2][0]), tr1 = v3(tmp[0][1], tmp[1][1], tmp[2][1]);
        V3 cr0 = v3(cov_c.c00, cov_c.c01, cov_c.c02), cr1 = v3(cov_c.c01, cov_c.c11, cov_c.c12),
           cr2 = v3(cov_c.c02, cov_c.c12, cov_c.c22);
        float vj00 = 2.0f * dot(tr0, cr0);
        float vj11 = 2.0f * dot(tr1, cr1);
        float vj20 = 2.0f * dot(tr0, cr2);
        float vj21 = 2.0f * dot(tr1, cr2);
        float txv = mz * mxc, tyv = mz * myc;
        if (in_x) v_mx += -u.fx * iz2 * vj20;
        else v_mz += -u.fx * iz3 * vj20 * txv;
        if (in_y) v_my += -u.fy * iz2 * vj21;
        else v_mz += -u.fy * iz3 * vj21 * tyv;
        v_mz += -u.fx * iz2 * vj00 - u.fy * iz2 * vj11 + 2.0f * u.fx * txv * iz3 * vj20 +
                2.0f * u.fy * tyv * iz3 * vj21;
        if (u.model != 0) {  // camera_model/mod.rs:88-136
            V3 g = u.model == 1 ? cam::kb4_vjp(J, mean_c, cov_c, intr_of(u), vcov, vmx, vmy)
                 : u.model == 2 ? cam::rt8_vjp(mean_c, cov_c, intr_of(u), vcov, vmx, vmy)
                                : cam::tpf_vjp(J, mean_c, cov_c, intr_of(u), vcov, vmx, vmy);
            v_mx = g.x;
            v_my = g.y;
            v_mz = g.z;
        }
        V3 v_mean_c = v3(v_mx, v_my, v_mz + vdep);
        // vcc = J^T v_cov2d J (Mat2x3::transpose_congruence_sym2, lib.rs:358-370)
        float sc[3][2];
        for (int c = 0; c < 3; ++c) {
            float jx = J.c[c][0], jy = J.c[c][1];
            sc[c][0] = vcov.c00 * jx + vcov.c01 * jy;
            sc[c][1] = vcov.c01 * jx + vcov.c11 * jy;
        }
        auto d2 = [&](int a, int b) { return J.c[a][0] * sc[b][0] + J.c[a][1] * sc[b][1]; };
        S3 vcc{d2(0, 0), d2(0, 1), d2(0, 2), d2(1, 1), d2(1, 2), d2(2, 2)};
        V3 v_mean = add(transpose_mul_vec3(u.rot, v_mean_c), v_mean_sh);
        // v_M = 2 * (R_view^T vcc R_view) * M (lib.rs:530-542, 494-512)
        V3 sc0 = s3mul(vcc, col(u.rot, 0)), sc1 = s3mul(vcc, col(u.rot, 1)), sc2 = s3mul(vcc, col(u.rot, 2));
        V3 q0 = col(u.rot, 0), q1 = col(u.rot, 1), q2 = col(u.rot, 2);
        S3 tc{dot(q0, sc0), dot(q0, sc1), dot(q0, sc2), dot(q1, sc1), dot(q1, sc2), dot(q2, sc2)};
        S3 tc2{tc.c00 * 2.0f, tc.c01 * 2.0f, tc.c02 * 2.0f, tc.c11 * 2.0f, tc.c12 * 2.0f, tc.c22 * 2.0f};
        M3 vM = from_cols(s3mul(tc2, col(Mm, 0)), s3mul(tc2, col(Mm, 1)), s3mul(tc2, col(Mm, 2)));
        V3 vse = v3(dot(col(R, 0), col(vM, 0)) * scl.x, dot(col(R, 1), col(vM, 1)) * scl.y,
                    dot(col(R, 2), col(vM, 2)) * scl.z);
        // quat_to_mat_vjp (project_backwards.rs:56-79) of v_M * diag(scale)
        M3 vr = mul_diag(vM, scl);
        float qw = q.w, qx = q.x, qy = q.y, qz = q.z;
        auto C = [&](int c, int r_) { return vr.c[c][r_]; };
        float wg = qx * (C(1, 2) - C(2, 1)) + qy * (C(2, 0) - C(0, 2)) + qz * (C(0, 1) - C(1, 0));
        float xg = -2.0f * qx * (C(1, 1) + C(2, 2)) + qy * (C(0, 1) + C(1, 0)) + qz * (C(0, 2) + C(2, 0)) +
                   qw * (C(1, 2) - C(2, 1));
        float yg = qx * (C(0, 1) + C(1, 0)) - 2.0f * qy * (C(0, 0) + C(2, 2)) + qz * (C(1, 2) + C(2, 1)) +
                   qw * (C(2, 0) - C(0, 2));
        float zg = qx * (C(0, 2) + C(2, 0)) + qy * (C(1, 2) + C(2, 1)) - 2.0f * qz * (C(0, 0) + C(1, 1)) +
                   qw * (C(0, 1) - C(1, 0));
        Q4 qg{2.0f * wg, 2.0f * xg, 2.0f * yg, 2.0f * zg};
        // apply_normalize_vjp (project_backwards.rs:20-52) on the raw quaternion
        float lsq = qdot(qu, qu);
        float l = std::sqrt(lsq);
        float inv = 1.0f / (l * lsq);
        float cc0 = -qu.w * qu.x, cc1 = -qu.x * qu.y, cc2 = -qu.y * qu.w;
        float cs0 = -qu.w * qu.z, cs1 = -qu.x * qu.z, cs2 = -qu.y * qu.z;
        float sw_ = qu.w * qu.w, sx_ = qu.x * qu.x, sy_ = qu.y * qu.y, sz_ = qu.z * qu.z;
        float vqw = ((lsq - sw_) * qg.w + cc0 * qg.x + cc2 * qg.y + cs0 * qg.z) * inv;
        float vqx = (cc0 * qg.w + (lsq - sx_) * qg.x + cc1 * qg.y + cs1 * qg.z) * inv;
        float vqy = (cc2 * qg.w + cc1 * qg.x + (lsq - sy_) * qg.y + cs2 * qg.z) * inv;
        float vqz = (cs0 * qg.w + cs1 * qg.x + cs2 * qg.y + (lsq - sz_) * qg.z) * inv;
        vt[0] = v_mean.x; vt[1] = v_mean.y; vt[2] = v_mean.z;
        vt[3] = vqw; vt[4] = vqx; vt[5] = vqy; vt[6] = vqz;
        vt[7] = vse.x; vt[8] = vse.y; vt[9] = vse.z;
    }
}

// 11-tap Gaussian (sigma 1.5) normalised, computed in float as the reference
// does at kernel-build time (brush-loss/src/lib.rs:87-100).
void orc_gauss_taps(float out[11]) {
    float s = 1.5f, sum = 0.0f;
    for (int i = 0; i < 11; ++i) {
        float x = (float)i - 5.0f;
        out[i] = std::exp(-x * x / (2.0f * s * s));
        sum += out[i];
    }
    for (int i = 0; i < 11; ++i) out[i] /= sum;
}

namespace {
const float kC1 = 0.01f * 0.01f;
const float kC2 = 0.03f * 0.03f;
const float kInv255 = 1.0f / 255.0f;

inline void read_gt(const uint32_t* gt, uint32_t c, size_t idx, float* gc, float* ga) {
    uint32_t v = gt[idx];
    *gc = (float)((v >> (c * 8u)) & 0xffu) * kInv255;
    *ga = (float)((v >> 24u) & 0xffu) * kInv255;
}

// Separable 11-tap blur with zero padding, reference summation order:
// sum over d = 1..5 of (left + right) * w[5-d], then the centre tap.
void blur_h(const std::vector<float>& src, std::vector<float>& dst, int W, int H, const float* w) {
#pragma omp parallel for schedule(static)
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            float s = 0.0f;
            for (int d = 1; d < 6; ++d) {
                float l = x - d >= 0 ? src[(size_t)y * W + x - d] : 0.0f;
                float r = x + d < W ? src[(size_t)y * W + x + d] : 0.0f;
                s += (l + r) * w[5 - d];
            }
            s += src[(size_t)y * W + x] * w[5];
            dst[(size_t)y * W + x] = s;
        }
}
void blur_v(const std::vector<float>& src, std::vector<float>& dst, int W, int H, const float* w) {
#pragma omp parallel for schedule(static)
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            float s = 0.0f;
            for (int d = 1; d < 6; ++d) {
                float t = y - d >= 0 ? src[(size_t)(y - d) * W + x] : 0.0f;
                float b = y + d < H ? src[(size_t)(y + d) * W + x] : 0.0f;
                s += (t + b) * w[5 - d];
            }
            s += src[(size_t)y * W + x] * w[5];
            dst[(size_t)y * W + x] = s;
        }
}

// The horizontal pass of the reference squares/multiplies inside the tap
// loop: sum_x2 += (xl*xl + xr*xr) * w. Restated directly for the 5 moments.
void blur_h_moments(const std::vector<float>& X, const std::vector<float>& Y, std::vector<float> out[5], int W, int H,
                    const float* w) {
    for (int k = 0; k < 5; ++k) out[k].assign((size_t)W * H, 0.0f);
#pragma omp parallel for schedule(static)
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            float sx = 0, sx2 = 0, sy = 0, sy2 = 0, sxy = 0;
            for (int d = 1; d < 6; ++d) {
                size_t il = (size_t)y * W + x - d, ir = (size_t)y * W + x + d;
                float xl = x - d >= 0 ? X[il] : 0.0f, yl = x - d >= 0 ? Y[il] : 0.0f;
                float xr = x + d < W ? X[ir] : 0.0f, yr = x + d < W ? Y[ir] : 0.0f;
                float wd = w[5 - d];
                sx += (xl + xr) * wd;
                sx2 += (xl * xl + xr * xr) * wd;
                sy += (yl + yr) * wd;
                sy2 += (yl * yl + yr * yr) * wd;
                sxy += (xl * yl + xr * yr) * wd;
            }
            size_t ic = (size_t)y * W + x;
            float xc = X[ic], yc = Y[ic], wc = w[5];
            sx += xc * wc;
            sx2 += xc * xc * wc;
            sy += yc * wc;
            sy2 += yc * yc * wc;
            sxy += xc * yc * wc;
            out[0][ic] = sx; out[1][ic] = sx2; out[2][ic] = sy; out[3][ic] = sy2; out[4][ic] = sxy;
        }
}

struct SsimTerms { float val, dmu1, dsig1, dsig12; };
// brush-loss/src/lib.rs:193-209 and :480-500
inline SsimTerms ssim_terms(const float o[5]) {
    float mu1 = o[0], mu2 = o[2];
    float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2;
    float s1 = bsx_max(0.0f, o[1] - mu1_sq);
    float s2 = bsx_max(0.0f, o[3] - mu2_sq);
    float s12 = o[4] - mu1 * mu2;
    float a = mu1_sq + mu2_sq + kC1;
    float b = s1 + s2 + kC2;
    float ct = 2.0f * mu1 * mu2 + kC1;
    float dt = 2.0f * s12 + kC2;
    SsimTerms t;
    float rawv = (ct * dt) / (a * b);
    t.val = bsx_clamp(rawv, -1.0f, 1.0f);
    float inv_ab = 1.0f / (a * b);
    float cd = ct * dt * inv_ab;
    bool clamped = cd < -1.0f || cd > 1.0f;
    t.dmu1 = clamped ? 0.0f : 2.0f * mu2 * inv_ab * (dt - ct) - 2.0f * mu1 * cd * (1.0f / a - 1.0f / b);
    t.dsig1 = clamped ? 0.0f : -cd / b;
    t.dsig12 = clamped ? 0.0f : 2.0f * ct * inv_ab;
    return t;
}

inline float gt_eff_of(const uint32_t* gt, uint32_t c, size_t idx, const bsx_loss_cfg* cfg, float* ga) {
    float gc;
    read_gt(gt, c, idx, &gc, ga);
    if (cfg->composite_bg) gc = gc + (1.0f - *ga) * cfg->bg[c];
    return gc;
}
}  // namespace

// Loss forward (brush-loss/src/lib.rs:354-542): pred/map are [C,H,W].
void orc_loss_fwd(const float* pred, const uint32_t* gt, uint32_t W, uint32_t H, uint32_t C,
                  const bsx_loss_cfg* cfg, float* map) {
    float w[11];
    orc_gauss_taps(w);
    const size_t P = (size_t)W * H;
    for (uint32_t c = 0; c < C; ++c) {
        if (c == 3) {
            for (size_t i = 0; i < P; ++i) {
                float gc, ga;
                read_gt(gt, 0, i, &gc, &ga);
                float v = std::fabs(pred[3 * P + i] - ga);
                if (cfg->mask) v = v * ga;
                map[3 * P + i] = v;
            }
            continue;
        }
        std::vector<float> X(pred + c * P, pred + (c + 1) * P), Y(P);
        for (size_t i = 0; i < P; ++i) {
            float ga;
            Y[i] = gt_eff_of(gt, c, i, cfg, &ga);
        }
        if (cfg->ssim_weight == 0.0f) {
            for (size_t i = 0; i < P; ++i) {
                float ga, gc = gt_eff_of(gt, c, i, cfg, &ga);
                float v = cfg->l1_weight * std::fabs(X[i] - gc);
                if (cfg->mask) v = v * ga;
                map[c * P + i] = v;
            }
            continue;
        }
        std::vector<float> hm[5], vm(P);
        blur_h_moments(X, Y, hm, (int)W, (int)H, w);
        std::vector<float> om[5];
        for (int k = 0; k < 5; ++k) {
            om[k].resize(P);
            blur_v(hm[k], om[k], (int)W, (int)H, w);
        }
        for (size_t i = 0; i < P; ++i) {
            float o[5] = {om[0][i], om[1][i], om[2][i], om[3][i], om[4][i]};
            SsimTerms t = ssim_terms(o);
            float l1 = std::fabs(X[i] - Y[i]);
            float v = cfg->l1_weight * l1 + cfg->ssim_weight * t.val;
            if (cfg->mask) {
                float gc, ga;
                read_gt(gt, c, i, &gc, &ga);
                v = v * ga;
            }
            map[c * P + i] = v;
        }
    }
}

// Loss backward (brush-loss/src/lib.rs:553-890): dl_dmap, dl_dpred are [C,H,W].
void orc_loss_bwd(const float* pred, const uint32_t* gt, uint32_t W, uint32_t H, uint32_t C,
                  const bsx_loss_cfg* cfg, const float* dl_dmap, float* dl_dpred) {
    float w[11];
    orc_gauss_taps(w);
    const size_t P = (size_t)W * H;
    for (uint32_t c = 0; c < C; ++c) {
        if (c == 3) {
            for (size_t i = 0; i < P; ++i) {
                float gc, ga;
                read_gt(gt, 0, i, &gc, &ga);
                float diff = pred[3 * P + i] - ga;
                float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
                float ch = dl_dmap[3 * P + i];
                if (cfg->mask) ch = ch * ga;
                dl_dpred[3 * P + i] = sign * ch;
            }
            continue;
        }
        std::vector<float> X(pred + c * P, pred + (c + 1) * P), Y(P);
        for (size_t i = 0; i < P; ++i) {
            float ga;
            Y[i] = gt_eff_of(gt, c, i, cfg, &ga);
        }
        if (cfg->ssim_weight == 0.0f) {
            for (size_t i = 0; i < P; ++i) {
                float diff = X[i] - Y[i];
                float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
                float ch = dl_dmap[c * P + i];
                if (cfg->mask) {
                    float gc, ga;
                    read_gt(gt, c, i, &gc, &ga);
                    ch = ch * ga;
                }
                dl_dpred[c * P + i] = cfg->l1_weight * sign * ch;
            }
            continue;
        }
        std::vector<float> hm[5];
        blur_h_moments(X, Y, hm, (int)W, (int)H, w);
        std::vector<float> om[5];
        for (int k = 0; k < 5; ++k) {
            om[k].resize(P);
            blur_v(hm[k], om[k], (int)W, (int)H, w);
        }
        std::vector<float> pa[3];
        for (int k = 0; k < 3; ++k) pa[k].assign(P, 0.0f);
        for (size_t i = 0; i < P; ++i) {
            float o[5] = {om[0][i], om[1][i], om[2][i], om[3][i], om[4][i]};
            SsimTerms t = ssim_terms(o);
            float ch = dl_dmap[c * P + i];
            if (cfg->mask) {
                float gc, ga;
                read_gt(gt, c, i, &gc, &ga);
                ch = ch * ga;
            }
            pa[0][i] = t.dmu1 * ch;
            pa[1][i] = t.dsig1 * ch;
            pa[2][i] = t.dsig12 * ch;
        }
        std::vector<float> h[3], s[3];
        for (int k = 0; k < 3; ++k) {
            h[k].resize(P);
            s[k].resize(P);
            blur_h(pa[k], h[k], (int)W, (int)H, w);
            blur_v(h[k], s[k], (int)W, (int)H, w);
        }
        for (size_t i = 0; i < P; ++i) {
            float p1 = X[i];
            float ga, ge = gt_eff_of(gt, c, i, cfg, &ga);
            float sg = s[0][i] + (2.0f * p1) * s[1][i] + ge * s[2][i];
            float diff = p1 - ge;
            float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            float chc = dl_dmap[c * P + i];
            if (cfg->mask) chc = chc * ga;
            dl_dpred[c * P + i] = cfg->ssim_weight * sg + cfg->l1_weight * sign * chc;
        }
    }
}

// AdamScaled::step for one parameter tensor (adam_scaled.rs:216-383).
// m/v updated in place; bias corrections use powi in float.
void orc_adam(float* param, const float* grad_in, float* m, float* v, uint32_t rows, uint32_t cols, float lr,
              const float* col_scale, int reduce, float beta1, float beta2, float eps, uint32_t step,
              float grad_scale) {
    auto powi = [](float b, uint32_t e) {
        float r = 1.0f;
        for (uint32_t i = 0; i < e; ++i) r *= b;
        return r;
    };
    float bc1 = 1.0f - powi(beta1, step);
    float bc2 = 1.0f - powi(beta2, step);
    bool first = step == 1;
#pragma omp parallel for schedule(static)
    for (int64_t ri = 0; ri < (int64_t)rows; ++ri) {
        size_t r0 = (size_t)ri * cols;
        float vr = 0.0f;
        if (reduce) {
            float s = 0.0f;
            for (uint32_t c = 0; c < cols; ++c) {
                float g = grad_in[r0 + c] * grad_scale;
                s += g * g;
            }
            float gsq = s / (float)cols;
            vr = first ? gsq * (1.0f - beta2) : v[ri] * beta2 + gsq * (1.0f - beta2);
            v[ri] = vr;
        }
        for (uint32_t c = 0; c < cols; ++c) {
            float g = grad_in[r0 + c] * grad_scale;
            float mm = first ? g * (1.0f - beta1) : m[r0 + c] * beta1 + g * (1.0f - beta1);
            m[r0 + c] = mm;
            float vv;
            if (reduce) {
                vv = vr;
            } else {
                float gsq = g * g;
                vv = first ? gsq * (1.0f - beta2) : v[r0 + c] * beta2 + gsq * (1.0f - beta2);
                v[r0 + c] = vv;
            }
            float upd = (mm / bc1) / (std::sqrt(vv / bc2) + eps);
            float s = col_scale ? col_scale[c] * lr : lr;
            param[r0 + c] = param[r0 + c] - upd * s;
        }
    }
}

// Stable argsort on key & mask(ceil4(bits)) (brush-sort/src/lib.rs:16-129).
void orc_radix_argsort_u32(const uint32_t* keys, const uint32_t* vals, uint32_t n, uint32_t bits, uint32_t* ko,
                           uint32_t* vo) {
    uint32_t eff = (bits + 3) / 4 * 4;
    uint32_t mask = eff >= 32 ? 0xffffffffu : ((1u << eff) - 1u);
    std::vector<uint32_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0u);
    std::stable_sort(idx.begin(), idx.end(), [&](uint32_t a, uint32_t b) { return (keys[a] & mask) < (keys[b] & mask); });
    for (uint32_t i = 0; i < n; ++i) {
        ko[i] = keys[idx[i]];
        vo[i] = vals[idx[i]];
    }
}

void orc_prefix_sum_u32(const uint32_t* in, uint32_t n, uint32_t* out) {
    uint32_t acc = 0;
    for (uint32_t i = 0; i < n; ++i) {
        acc += in[i];
        out[i] = acc;
    }
}

void orc_tile_offsets(const uint32_t* ids, uint32_t n, uint32_t num_tiles, uint32_t* off) {
    std::memset(off, 0, sizeof(uint32_t) * (size_t)num_tiles * 2);
    for (uint32_t k = 0; k < n; ++k) {
        uint32_t tid = ids[k];
        if (k == 0) {
            if (tid < num_tiles) off[tid * 2] = 0;
        } else {
            uint32_t prev = ids[k - 1];
            if (tid != prev) {
                if (prev < num_tiles) off[prev * 2 + 1] = k;
                if (tid < num_tiles) off[tid * 2] = k;
            }
        }
        if (k == n - 1 && tid < num_tiles) off[tid * 2 + 1] = k + 1;
    }
}

// Global-order rasterizer with no spatial bins: every pixel composites all
// projected rows in the given order. Restates the reference's CPU raster
// oracle (crates/brush-render/src/tests/raster_oracle.rs:49-98); rows use the
// reference's 10-lane layout. Output [H,W,4].
void orc_rasterize_rows(const float* rows10, uint32_t count, uint32_t w, uint32_t h, const float bg[3], int smooth,
                        float* image) {
    for (uint32_t y = 0; y < h; ++y)
        for (uint32_t x = 0; x < w; ++x) {
            float pcx = (float)x + 0.5f, pcy = (float)y + 0.5f;
            float T_acc = 1.0f, r = 0.0f, g = 0.0f, b = 0.0f;
            for (uint32_t k = 0; k < count; ++k) {
                const float* s = rows10 + (size_t)k * 10;
                float dx = pcx - s[0], dy = pcy - s[1];
                float sigma = 0.5f * (s[2] * dx * dx + s[4] * dy * dy) + s[3] * dx * dy;
                float alpha = bsx_min(s[5] * bsx_expf(-sigma), 0.999f);
                float wgt = smooth ? alpha_cutoff_weight(alpha) : (alpha >= kCutMid ? 1.0f : 0.0f);
                if (sigma >= 0.0f && wgt > 0.0f) {
                    float ae = alpha * wgt;
                    float next_t = T_acc * (1.0f - ae);
                    if (next_t <= 1.0e-4f) break;
                    float v = ae * T_acc;
                    r += bsx_max(s[6], 0.0f) * v;
                    g += bsx_max(s[7], 0.0f) * v;
                    b += bsx_max(s[8], 0.0f) * v;
                    T_acc = next_t;
                }
            }
            float* o = image + ((size_t)y * w + x) * 4;
            o[0] = r + bg[0] * T_acc;
            o[1] = g + bg[1] * T_acc;
            o[2] = b + bg[2] * T_acc;
            o[3] = 1.0f - T_acc;
        }
}

// Deterministic float32 exp / ln used on both processors (exposed for tests).
float orc_expf(float x) { return bsx_expf(x); }
float orc_raster_sigma(float c00, float c01, float c11, float dx, float dy) {
    return bsx_raster_sigma(c00, c01, c11, dx, dy);
}
float orc_logf(float x) { return bsx_logf(x); }
float orc_atan2f(float y, float x) { return bsx_atan2f(y, x); }

// Largest error in ulp of the rasterizers' bsx_expf_raster against the
// exponential evaluated in double precision, over every `stride`-th float in
// [lo, 0] (lo <= 0, bit patterns from -0 downwards); -1 if any result is not
// finite and positive.
double orc_expf_raster_max_ulp(float lo, uint32_t stride) {
    const uint32_t last = bsx_f32_to_bits(-fabsf(lo));
    const int64_t step = stride ? stride : 1;
    double worst = 0.0;
#pragma omp parallel for reduction(max : worst) schedule(static)
    for (int64_t b = 0x80000000ll; b <= (int64_t)last; b += step) {
        const float x = bsx_bits_to_f32((uint32_t)b);
        const float y = bsx_expf_raster(x);
        const double ref = exp((double)x);
        if (!(y > 0.0f) || !bsx_is_finite(y)) {
            worst = 1e30;
            continue;
        }
        const double ulp = ldexp(1.0, ilogbf((float)ref) - 23);
        worst = fmax(worst, fabs((double)y - ref) / ulp);
    }
    return worst >= 1e30 ? -1.0 : worst;
}

void orc_set_raster_expr(int mode) { g_raster_expr = mode ? 1 : 0; }

// The mean-noise injection after the optimizer step (train.rs:1095-1169), in the
// reference's tensor order over every splat: inv = 1 - sigmoid(raw);
// noise_weight = clamp(inv^150, 0, 1) * gate (gate = 1 where d_gate > 0);
// noise_weight_means = noise_weight * scale (scale = f32(lr_mean) *
// mean_noise_weight); means += clamp(n * noise_weight_means, -limit, limit).
// The normals n are bsx_normal3(seed, step, i) (the library's counter-based
// generator; the reference draws from its device RNG).
void orc_mean_noise_step(float* transforms, const float* raw_opac, const float* gate, uint32_t n, float scale,
                         float limit, uint64_t seed, uint32_t step) {
#pragma omp parallel for schedule(static)
    for (int64_t gi = 0; gi < (int64_t)n; ++gi) {
        const uint32_t i = (uint32_t)gi;
        const float inv = 1.0f - bsx_sigmoid(raw_opac[i]);
        const float nw = bsx_clamp(bsx_powi(inv, 150u), 0.0f, 1.0f) * (gate[i] > 0.0f ? 1.0f : 0.0f);
        const float nwm = nw * scale;
        float z[3];
        bsx_normal3(seed, step, i, z);
        for (int k = 0; k < 3; ++k) transforms[(size_t)i * 10 + k] += bsx_clamp(z[k] * nwm, -limit, limit);
    }
}

void orc_sincos_2pi(float u, float* s, float* c) { bsx_sincos_2pi(u, s, c); }
// Largest |error| of bsx_sincos_2pi over every u = k / 2^24 (the generator's
// uniforms) against the double-precision sin / cos: out = {sin, cos}.
void orc_sincos_2pi_max_err(double out[2]) {
    double es = 0.0, ec = 0.0;
#pragma omp parallel for schedule(static) reduction(max : es, ec)
    for (int64_t k = 0; k < (1 << 24); ++k) {
        const float u = (float)k * 5.9604644775390625e-08f;
        float sn, cs;
        bsx_sincos_2pi(u, &sn, &cs);
        const double a = 6.283185307179586 * (double)u;
        es = std::max(es, std::fabs((double)sn - std::sin(a)));
        ec = std::max(ec, std::fabs((double)cs - std::cos(a)));
    }
    out[0] = es;
    out[1] = ec;
}
void orc_normal3_many(uint64_t seed, uint32_t step, uint32_t n, float* z) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) bsx_normal3(seed, step, (uint32_t)i, z + 3 * i);
}
void orc_normal3(uint64_t seed, uint32_t step, uint32_t index, float* z) { bsx_normal3(seed, step, index, z); }
float orc_powi(float b, uint32_t e) { return bsx_powi(b, e); }

// Decision flips between the two raster arithmetics along one render's
// trajectory: every pixel walks its tile's whole intersection run (the
// unshortened range) with the state of the render's own arithmetic, and at
// each pair evaluates both forms. out = {pairs walked, accept flips (sigma >= 0
// and alpha >= 1/255 differ), early-out flips (both accept; T (1 - alpha) <=
// 1e-4 differs), pixels}. Hard alpha cutoff only.
void orc_raster_decision_flips(void* h, uint64_t out[4]) {
    Render* r = (Render*)h;
    const Uni u = uni_from(r->uni);
    const uint32_t W = u.w, H = u.h, T = u.tbw * u.tbh, M = r->num_intersections;
    const int mode = r->raster_expr;
    std::vector<uint32_t> lo(T, 0), hi(T, 0);
    for (uint32_t k = 0; k < M; ++k) {
        const uint32_t t = r->isect_tile[k];
        if (t >= T) continue;
        if (k == 0 || r->isect_tile[k - 1] != t) lo[t] = k;
        hi[t] = k + 1;
    }
    uint64_t pairs = 0, acc_flip = 0, eo_flip = 0, pixels = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : pairs, acc_flip, eo_flip, pixels)
    for (int64_t ti = 0; ti < (int64_t)T; ++ti) {
        const uint32_t tile = (uint32_t)ti, tx = tile % u.tbw, ty = tile / u.tbw;
        for (uint32_t py = ty * 16; py < ty * 16 + 16; ++py)
            for (uint32_t px = tx * 16; px < tx * 16 + 16; ++px) {
                if (!(px < W && py < H)) continue;
                ++pixels;
                const float pcx = (float)px + 0.5f, pcy = (float)py + 0.5f;
                float T_acc = 1.0f;
                for (uint32_t k = lo[tile]; k < hi[tile]; ++k) {
                    const float* p = &r->projected[(size_t)r->isect_gid[k] * 12];
                    bool acc[2], eo[2];
                    float ae[2];
                    for (int m = 0; m < 2; ++m) {
                        const float sg = raster_sigma_mode(m, p[2], p[3], p[4], pcx - p[0], pcy - p[1]);
                        const float al = bsx_min(0.999f, p[5] * raster_gauss_mode(m, sg));
                        acc[m] = sg >= 0.0f && al >= kCutMid;
                        ae[m] = al;
                        eo[m] = T_acc * (1.0f - al) <= 1.0e-4f;
                    }
                    ++pairs;
                    if (acc[0] != acc[1]) ++acc_flip;
                    else if (acc[0] && eo[0] != eo[1]) ++eo_flip;
                    if (!acc[mode]) continue;
                    if (eo[mode]) break;
                    T_acc = T_acc * (1.0f - ae[mode]);
                }
            }
    }
    out[0] = pairs;
    out[1] = acc_flip;
    out[2] = eo_flip;
    out[3] = pixels;
}

}  // extern "C"
