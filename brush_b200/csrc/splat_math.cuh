// splat_math.cuh - device-side float32 geometry for projection, emission and
// projection backward. Operation order follows the reference's cube math so
// that results are reproducible bit-for-bit by a host restatement compiled
// without contraction; this file is compiled with -fmad=false.
//
// Reference: crates/brush-cube/src/lib.rs:39-638,
//            crates/brush-render/src/kernels/helpers.rs:86-363,
//            crates/brush-render/src/kernels/camera_model/pinhole.rs:24-123.
#pragma once
#include "common.cuh"

namespace bsx {

struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };
struct M3 { V3 c0, c1, c2; };  // columns
struct S2 { float c00, c01, c11; };
struct S3 { float c00, c01, c02, c11, c12, c22; };
struct M23 { float c0x, c0y, c1x, c1y, c2x, c2y; };

__device__ __forceinline__ V3 v3(float x, float y, float z) { return V3{x, y, z}; }
__device__ __forceinline__ V3 vadd(V3 a, V3 b) { return v3(a.x + b.x, a.y + b.y, a.z + b.z); }
__device__ __forceinline__ V3 vsub(V3 a, V3 b) { return v3(a.x - b.x, a.y - b.y, a.z - b.z); }
__device__ __forceinline__ V3 vscale(V3 a, float s) { return v3(a.x * s, a.y * s, a.z * s); }
__device__ __forceinline__ float vdot(V3 a, V3 b) { return (a.x * b.x + a.y * b.y) + a.z * b.z; }
__device__ __forceinline__ bool vfinite(V3 a) { return bsx_is_finite(a.x) && bsx_is_finite(a.y) && bsx_is_finite(a.z); }
__device__ __forceinline__ V3 mrow(const M3& m, int i) {
    return i == 0 ? v3(m.c0.x, m.c1.x, m.c2.x) : (i == 1 ? v3(m.c0.y, m.c1.y, m.c2.y) : v3(m.c0.z, m.c1.z, m.c2.z));
}
// M * v = (c0*x + c1*y) + c2*z
__device__ __forceinline__ V3 mmul(const M3& m, V3 v) { return vadd(vadd(vscale(m.c0, v.x), vscale(m.c1, v.y)), vscale(m.c2, v.z)); }
__device__ __forceinline__ V3 mtmul(const M3& m, V3 v) { return v3(vdot(m.c0, v), vdot(m.c1, v), vdot(m.c2, v)); }
__device__ __forceinline__ M3 mmulm(const M3& m, const M3& n) { return M3{mmul(m, n.c0), mmul(m, n.c1), mmul(m, n.c2)}; }
__device__ __forceinline__ M3 mdiag(const M3& m, V3 s) { return M3{vscale(m.c0, s.x), vscale(m.c1, s.y), vscale(m.c2, s.z)}; }

__device__ __forceinline__ float qdot(Q4 a, Q4 b) { return ((a.w * b.w + a.x * b.x) + a.y * b.y) + a.z * b.z; }
__device__ __forceinline__ Q4 qnormalize(Q4 q) {
    float s = 1.0f / sqrtf(qdot(q, q));
    return Q4{q.w * s, q.x * s, q.y * s, q.z * s};
}
// Quat::to_mat3 (lib.rs:191-216)
__device__ __forceinline__ M3 quat_to_mat3(Q4 q) {
    float x2 = q.x * q.x, y2 = q.y * q.y, z2 = q.z * q.z;
    float xy = q.x * q.y, xz = q.x * q.z, yz = q.y * q.z;
    float wx = q.w * q.x, wy = q.w * q.y, wz = q.w * q.z;
    return M3{v3(1.0f - 2.0f * (y2 + z2), 2.0f * (xy + wz), 2.0f * (xz - wy)),
              v3(2.0f * (xy - wz), 1.0f - 2.0f * (x2 + z2), 2.0f * (yz + wx)),
              v3(2.0f * (xz + wy), 2.0f * (yz - wx), 1.0f - 2.0f * (x2 + y2))};
}

__device__ __forceinline__ S2 sym2_inverse(S2 m) {
    float det = m.c00 * m.c11 - m.c01 * m.c01;
    float inv_det = det > 0.0f ? 1.0f / det : 0.0f;
    return S2{m.c11 * inv_det, -m.c01 * inv_det, m.c00 * inv_det};
}
__device__ __forceinline__ float det2_strict(S2 m) {
    float ad = m.c00 * m.c11;
    float bc = m.c01 * m.c01;
    return ad - bc;
}
__device__ __forceinline__ bool s2finite(S2 m) {
    return bsx_is_finite(m.c00) && bsx_is_finite(m.c11) && bsx_is_finite(m.c01);
}
// calc_sigma (lib.rs:634-638)
__device__ __forceinline__ float calc_sigma(float px, float py, float c00, float c01, float c11, float x, float y) {
    float dx = px - x;
    float dy = py - y;
    return 0.5f * (c00 * dx * dx + c11 * dy * dy) + c01 * dx * dy;
}

// Uniforms as the kernels consume them.
struct Uni {
    M3 rot;
    V3 trans;
    float fx, fy, cx, cy;
    float lpx, lpy, lnx, lny;
    V3 cam;
    uint32_t w, h, tbw, tbh;
    float half_max_fov;
    int model;       // bsx_camera_model
    float kp[BSX_CAMERA_PARAMS];
};

inline Uni make_uni(const bsx_project_uniforms& u) {
    Uni r;
    const float* m = u.viewmat;
    r.rot.c0 = V3{m[0], m[1], m[2]};
    r.rot.c1 = V3{m[3], m[4], m[5]};
    r.rot.c2 = V3{m[6], m[7], m[8]};
    r.trans = V3{m[9], m[10], m[11]};
    r.fx = u.fx; r.fy = u.fy; r.cx = u.cx; r.cy = u.cy;
    r.lpx = u.lim_pos_x; r.lpy = u.lim_pos_y; r.lnx = u.lim_neg_x; r.lny = u.lim_neg_y;
    r.cam = V3{u.camera_pos[0], u.camera_pos[1], u.camera_pos[2]};
    r.w = u.img_w; r.h = u.img_h; r.tbw = u.tile_bw; r.tbh = u.tile_bh;
    r.half_max_fov = u.half_max_render_fov;
    r.model = u.camera_model;
    for (int k = 0; k < BSX_CAMERA_PARAMS; ++k) r.kp[k] = u.model_params[k];
    return r;
}

// Pinhole Jacobian with clamped normalised coordinates (pinhole.rs:31-56).
__device__ __forceinline__ M23 pinhole_jacobian(V3 p, const Uni& u) {
    float inv_z = 1.0f / p.z;
    float dx = u.fx * inv_z;
    float dy = u.fy * inv_z;
    float cx = bsx_clamp(p.x * inv_z, u.lnx, u.lpx);
    float cy = bsx_clamp(p.y * inv_z, u.lny, u.lpy);
    return M23{dx, 0.0f, 0.0f, dy, -dx * cx, -dy * cy};
}

__device__ __forceinline__ M23 project_jacobian(V3 p, const Uni& u);  // camera_models.cuh

// calc_cov2d (helpers.rs:297-330) with the camera model's projection Jacobian
__device__ __forceinline__ S2 calc_cov2d(V3 scl, Q4 q, V3 mean_c, const Uni& u) {
    M3 ns = mdiag(mmulm(u.rot, quat_to_mat3(q)), scl);
    M23 j = project_jacobian(mean_c, u);
    // V = J * ns, column i = (J.c0*n.x + J.c1*n.y) + J.c2*n.z
    float v0x = (j.c0x * ns.c0.x + j.c1x * ns.c0.y) + j.c2x * ns.c0.z;
    float v0y = (j.c0y * ns.c0.x + j.c1y * ns.c0.y) + j.c2y * ns.c0.z;
    float v1x = (j.c0x * ns.c1.x + j.c1x * ns.c1.y) + j.c2x * ns.c1.z;
    float v1y = (j.c0y * ns.c1.x + j.c1y * ns.c1.y) + j.c2y * ns.c1.z;
    float v2x = (j.c0x * ns.c2.x + j.c1x * ns.c2.y) + j.c2x * ns.c2.z;
    float v2y = (j.c0y * ns.c2.x + j.c1y * ns.c2.y) + j.c2y * ns.c2.z;
    float c00 = (v0x * v0x + v1x * v1x) + v2x * v2x;
    float c01 = (v0x * v0y + v1x * v1y) + v2x * v2y;
    float c11 = (v0y * v0y + v1y * v1y) + v2y * v2y;
    const float lim = 1.0e18f;
    float max_abs = bsx_max(bsx_max(fabsf(c00), fabsf(c11)), fabsf(c01));
    float sd = max_abs > lim ? lim / max_abs : 1.0f;
    return S2{c00 * sd, c01 * sd, c11 * sd};
}

// compensate_cov2d (helpers.rs:335-350)
__device__ __forceinline__ S2 compensate_cov2d(S2 c, bool mip, float* filter_comp) {
    float blur = mip ? 0.1f : 0.3f;
    S2 b{c.c00 + blur, c.c01, c.c11 + blur};
    float fc = 1.0f;
    if (mip) {
        float det_raw = bsx_max(det2_strict(c), 0.0f);
        float det_b = det2_strict(b);
        fc = sqrtf(det_raw / det_b);
    }
    *filter_comp = fc;
    return b;
}

// compute_bbox_extent (helpers.rs:230-241)
__device__ __forceinline__ void bbox_extent(S2 conic, float pt, float* ex, float* ey) {
    float det = conic.c00 * conic.c11 - conic.c01 * conic.c01;
    bool degenerate = det <= 0.0f;
    float inv_det = degenerate ? 0.0f : 1.0f / det;
    float x = sqrtf(2.0f * pt * conic.c11 * inv_det);
    float y = sqrtf(2.0f * pt * conic.c00 * inv_det);
    *ex = degenerate ? -1.0f : x;
    *ey = degenerate ? -1.0f : y;
}

struct TileBox { uint32_t min_x, min_y, max_x, max_y; };
// get_tile_bbox (helpers.rs:262-295)
__device__ __forceinline__ TileBox tile_bbox(float cx, float cy, float ex, float ey, uint32_t bw, uint32_t bh) {
    float pcx = cx / 16.0f, pcy = cy / 16.0f, dx = ex / 16.0f, dy = ey / 16.0f;
    float bwf = (float)bw, bhf = (float)bh;
    TileBox b;
    b.min_x = (uint32_t)bsx_clamp(pcx - dx, 0.0f, bwf);
    b.min_y = (uint32_t)bsx_clamp(pcy - dy, 0.0f, bhf);
    b.max_x = (uint32_t)bsx_clamp(pcx + dx + 1.0f, 0.0f, bwf);
    b.max_y = (uint32_t)bsx_clamp(pcy + dy + 1.0f, 0.0f, bhf);
    return b;
}

// will_primitive_contribute (helpers.rs:385-424), StopThePop tile test.
__device__ __forceinline__ bool tile_contrib(uint32_t tx, uint32_t ty, float mx, float my, S2 conic, float pt) {
    float rminx = (float)(tx * 16u), rminy = (float)(ty * 16u);
    float rmaxx = rminx + 16.0f, rmaxy = rminy + 16.0f;
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
        float txc = in_y ? 0.0f : bsx_clamp(tx_raw, 0.0f, 1.0f);
        float tyc = in_x ? 0.0f : bsx_clamp(ty_raw, 0.0f, 1.0f);
        float max_x = corner_x + txc * dxf;
        float max_y = corner_y + tyc * dyf;
        hit = calc_sigma(max_x, max_y, conic.c00, conic.c01, conic.c11, mx, my) <= pt;
    }
    return hit;
}

}  // namespace bsx

#include "camera_models.cuh"
