// camera_models.cuh - projection, projection Jacobian and projection VJP per
// camera model, restating crates/brush-render/src/kernels/camera_model/
// (pinhole.rs:24-123, kannala_brandt_4.rs:18-337, radial_tangential_8.rs:22-377,
// thin_prism_fisheye.rs:31-203) operation for operation (this file is
// compiled without contraction; atan2 is the shared deterministic bsx_atan2f),
// so a CPU restatement reproduces every bit. The model is a launch uniform:
// every branch on it is uniform across the grid.
#pragma once
#include "splat_math.cuh"

namespace bsx {

// ---- pinhole -----------------------------------------------------------------
__device__ __forceinline__ void project_pinhole(V3 p, const Uni& u, float* px, float* py) {
    const float inv_z = 1.0f / p.z;
    *px = u.fx * p.x * inv_z + u.cx;
    *py = u.fy * p.y * inv_z + u.cy;
}

// ---- Kannala-Brandt 4 ----------------------------------------------------------
__device__ __forceinline__ void project_kb4(V3 p, const Uni& u, const float* k, float* px, float* py) {
    const float x = p.x, y = p.y, z = p.z;
    const float inv_z = 1.0f / z;
    const float pin_u = u.fx * x * inv_z + u.cx;
    const float pin_v = u.fy * y * inv_z + u.cy;
    const float r = sqrtf(x * x + y * y);
    const float theta = bsx_atan2f(r, z);
    const float t2 = theta * theta, t4 = t2 * t2, t6 = t2 * t4, t8 = t4 * t4;
    const float d = theta * (1.0f + k[0] * t2 + k[1] * t4 + k[2] * t6 + k[3] * t8);
    const float inv_r = 1.0f / r;
    const float fu = u.fx * (d * x * inv_r) + u.cx;
    const float fv = u.fy * (d * y * inv_r) + u.cy;
    const bool near_axis = r < 1e-6f;
    *px = near_axis ? pin_u : fu;
    *py = near_axis ? pin_v : fv;
}

__device__ __forceinline__ M23 jacobian_kb4(V3 p, const Uni& u, const float* k) {
    const float fx = u.fx, fy = u.fy;
    const float x = p.x, y = p.y, z = p.z;
    const float inv_z = 1.0f / z;
    const float x2 = x * x, y2 = y * y, xy = x * y;
    const float r2 = x2 + y2;
    const float r = sqrtf(r2);
    const float inv_r = 1.0f / r;
    const float inv_r3 = inv_r * inv_r * inv_r;
    const float rho2 = r2 + z * z;
    const float inv_rho2 = 1.0f / rho2;
    const float inv_rho2_r = inv_rho2 * inv_r;
    const float theta = bsx_atan2f(r, z);
    const float t2 = theta * theta, t4 = t2 * t2, t6 = t4 * t2, t8 = t4 * t4;
    const float d = theta * (1.0f + k[0] * t2 + k[1] * t4 + k[2] * t6 + k[3] * t8);
    const float dd = 1.0f + 3.0f * k[0] * t2 + 5.0f * k[1] * t4 + 7.0f * k[2] * t6 + 9.0f * k[3] * t8;
    const float dth_dx = x * z * inv_rho2_r, dth_dy = y * z * inv_rho2_r, dth_dz = -r * inv_rho2;
    const float dd_dx = dd * dth_dx, dd_dy = dd * dth_dy, dd_dz = dd * dth_dz;
    const float xr = x * inv_r;
    const float dxr_dx = y2 * inv_r3, dxr_dy = -xy * inv_r3;
    const float du_dx = fx * (dd_dx * xr + d * dxr_dx);
    const float du_dy = fx * (dd_dy * xr + d * dxr_dy);
    const float du_dz = fx * (dd_dz * xr);
    const float yr = y * inv_r;
    const float dyr_dx = -xy * inv_r3, dyr_dy = x2 * inv_r3;
    const float dv_dx = fy * (dd_dx * yr + d * dyr_dx);
    const float dv_dy = fy * (dd_dy * yr + d * dyr_dy);
    const float dv_dz = fy * (dd_dz * yr);
    const bool near_axis = r < 1e-6f;
    const float dx = fx * inv_z, dy = fy * inv_z;
    const float p_du_dz = -dx * x * inv_z, p_dv_dz = -dy * y * inv_z;
    return M23{near_axis ? dx : du_dx,   near_axis ? 0.0f : dv_dx,  near_axis ? 0.0f : du_dy,
               near_axis ? dy : dv_dy,   near_axis ? p_du_dz : du_dz, near_axis ? p_dv_dz : dv_dz};
}

// Rows of 2 * (v_cov2d J) cov_c, as the reference forms them (Sym2::mul_mat2x3, row dots).
struct VJRows {
    float u0, u1, u2, v0, v1, v2;
};
__device__ __forceinline__ VJRows vj_rows(const M23& J, S2 vc, const S3& cc) {
    const float t0x = vc.c00 * J.c0x + vc.c01 * J.c0y, t0y = vc.c01 * J.c0x + vc.c11 * J.c0y;
    const float t1x = vc.c00 * J.c1x + vc.c01 * J.c1y, t1y = vc.c01 * J.c1x + vc.c11 * J.c1y;
    const float t2x = vc.c00 * J.c2x + vc.c01 * J.c2y, t2y = vc.c01 * J.c2x + vc.c11 * J.c2y;
    const V3 r0 = v3(t0x, t1x, t2x), r1 = v3(t0y, t1y, t2y);
    const V3 c0 = v3(cc.c00, cc.c01, cc.c02), c1 = v3(cc.c01, cc.c11, cc.c12), c2 = v3(cc.c02, cc.c12, cc.c22);
    return VJRows{2.0f * vdot(r0, c0), 2.0f * vdot(r0, c1), 2.0f * vdot(r0, c2),
                  2.0f * vdot(r1, c0), 2.0f * vdot(r1, c1), 2.0f * vdot(r1, c2)};
}

__device__ __forceinline__ V3 vjp_kb4(const M23& J, V3 mc, const S3& cc, const Uni& u, S2 vcov, float vmx,
                                      float vmy, const float* k) {
    const float fx = u.fx, fy = u.fy;
    const float mx = mc.x, my = mc.y, mz = mc.z;
    const float r2 = mx * mx + my * my;
    const float r = fmaxf(sqrtf(r2), 1.0e-8f);
    const float rho2 = r2 + mz * mz;
    const float theta = bsx_atan2f(r, mz);
    const float th2 = theta * theta, th4 = th2 * th2, th6 = th4 * th2, th8 = th4 * th4;
    const float theta_d = theta * (1.0f + k[0] * th2 + k[1] * th4 + k[2] * th6 + k[3] * th8);
    const float p1 = 1.0f + 3.0f * k[0] * th2 + 5.0f * k[1] * th4 + 7.0f * k[2] * th6 + 9.0f * k[3] * th8;
    const float p2 = 6.0f * k[0] * theta + 20.0f * k[1] * theta * th2 + 42.0f * k[2] * theta * th4 +
                     72.0f * k[3] * theta * th6;
    const float inv_r = 1.0f / r;
    const float inv_r3 = inv_r * inv_r * inv_r;
    const float inv_r5 = inv_r3 * inv_r * inv_r;
    const float inv_rho2 = 1.0f / rho2;
    const float inv_rho2_sq = inv_rho2 * inv_rho2;
    const float inv_rho2_r = inv_rho2 * inv_r;
    const float dth_x = mx * mz * inv_rho2_r, dth_y = my * mz * inv_rho2_r, dth_z = -r * inv_rho2;
    const float xr = mx * inv_r, yr = my * inv_r;
    const float dxr_x = my * my * inv_r3, dxr_y = -mx * my * inv_r3;
    const float dyr_x = dxr_y, dyr_y = mx * mx * inv_r3;
    const float dg_x = p1 * dth_x, dg_y = p1 * dth_y, dg_z = p1 * dth_z;
    // path 1: J^T v_mean2d (Vec2::dot)
    float v_mx = vmx * J.c0x + vmy * J.c0y;
    float v_my = vmx * J.c1x + vmy * J.c1y;
    float v_mz = vmx * J.c2x + vmy * J.c2y;
    const VJRows vj = vj_rows(J, vcov, cc);
    // Hessians of theta and of x/r, y/r
    const float three_r2_z2 = 3.0f * r2 + mz * mz;
    const float r2_minus_z2 = r2 - mz * mz;
    const float h_th_00 = mz * (r2 * rho2 - mx * mx * three_r2_z2) * inv_r3 * inv_rho2_sq;
    const float h_th_11 = mz * (r2 * rho2 - my * my * three_r2_z2) * inv_r3 * inv_rho2_sq;
    const float h_th_01 = -mx * my * mz * three_r2_z2 * inv_r3 * inv_rho2_sq;
    const float h_th_02 = mx * r2_minus_z2 * inv_r * inv_rho2_sq;
    const float h_th_12 = my * r2_minus_z2 * inv_r * inv_rho2_sq;
    const float h_th_22 = 2.0f * mz * r * inv_rho2_sq;
    const float two_x2_my2 = 2.0f * mx * mx - my * my;
    const float two_y2_mx2 = 2.0f * my * my - mx * mx;
    const float h_xr_00 = -3.0f * mx * my * my * inv_r5;
    const float h_xr_01 = my * two_x2_my2 * inv_r5;
    const float h_xr_11 = mx * two_y2_mx2 * inv_r5;
    const float h_yr_00 = my * two_x2_my2 * inv_r5;
    const float h_yr_01 = mx * two_y2_mx2 * inv_r5;
    const float h_yr_11 = -3.0f * mx * mx * my * inv_r5;
    // path 2: contraction with the derivative of J
    {
        const float d2g = p2 * dth_x * dth_x + p1 * h_th_00;
        const float d_ju = fx * (d2g * xr + dg_x * dxr_x + dg_x * dxr_x + theta_d * h_xr_00);
        const float d_jv = fy * (d2g * yr + dg_x * dyr_x + dg_x * dyr_x + theta_d * h_yr_00);
        v_mx += vj.u0 * d_ju + vj.v0 * d_jv;
    }
    {
        const float d2g = p2 * dth_y * dth_x + p1 * h_th_01;
        const float d_ju = fx * (d2g * xr + dg_y * dxr_x + dg_x * dxr_y + theta_d * h_xr_01);
        const float d_jv = fy * (d2g * yr + dg_y * dyr_x + dg_x * dyr_y + theta_d * h_yr_01);
        v_mx += vj.u1 * d_ju + vj.v1 * d_jv;
    }
    {
        const float d2g = p2 * dth_z * dth_x + p1 * h_th_02;
        const float d_ju = fx * (d2g * xr + dg_x * 0.0f + dg_z * dxr_x);
        const float d_jv = fy * (d2g * yr + dg_x * 0.0f + dg_z * dyr_x);
        v_mx += vj.u2 * d_ju + vj.v2 * d_jv;
    }
    {
        const float d2g = p2 * dth_x * dth_y + p1 * h_th_01;
        const float d_ju = fx * (d2g * xr + dg_x * dxr_y + dg_y * dxr_x + theta_d * h_xr_01);
        const float d_jv = fy * (d2g * yr + dg_x * dyr_y + dg_y * dyr_x + theta_d * h_yr_01);
        v_my += vj.u0 * d_ju + vj.v0 * d_jv;
    }
    {
        const float d2g = p2 * dth_y * dth_y + p1 * h_th_11;
        const float d_ju = fx * (d2g * xr + dg_y * dxr_y + dg_y * dxr_y + theta_d * h_xr_11);
        const float d_jv = fy * (d2g * yr + dg_y * dyr_y + dg_y * dyr_y + theta_d * h_yr_11);
        v_my += vj.u1 * d_ju + vj.v1 * d_jv;
    }
    {
        const float d2g = p2 * dth_z * dth_y + p1 * h_th_12;
        const float d_ju = fx * (d2g * xr + dg_y * 0.0f + dg_z * dxr_y);
        const float d_jv = fy * (d2g * yr + dg_y * 0.0f + dg_z * dyr_y);
        v_my += vj.u2 * d_ju + vj.v2 * d_jv;
    }
    {
        const float d2g = p2 * dth_x * dth_z + p1 * h_th_02;
        const float d_ju = fx * (d2g * xr + dg_z * dxr_x + dg_x * 0.0f);
        const float d_jv = fy * (d2g * yr + dg_z * dyr_x + dg_x * 0.0f);
        v_mz += vj.u0 * d_ju + vj.v0 * d_jv;
    }
    {
        const float d2g = p2 * dth_y * dth_z + p1 * h_th_12;
        const float d_ju = fx * (d2g * xr + dg_z * dxr_y + dg_y * 0.0f);
        const float d_jv = fy * (d2g * yr + dg_z * dyr_y + dg_y * 0.0f);
        v_mz += vj.u1 * d_ju + vj.v1 * d_jv;
    }
    {
        const float d2g = p2 * dth_z * dth_z + p1 * h_th_22;
        const float d_ju = fx * (d2g * xr);
        const float d_jv = fy * (d2g * yr);
        v_mz += vj.u2 * d_ju + vj.v2 * d_jv;
    }
    return v3(v_mx, v_my, v_mz);
}

// ---- radial-tangential 8 ---------------------------------------------------------
__device__ __forceinline__ void project_rt8(V3 p, const Uni& u, const float* k, float* px, float* py) {
    const float x_ = p.x / p.z, y_ = p.y / p.z;
    const float x_2 = x_ * x_, y_2 = y_ * y_;
    const float r2 = x_2 + y_2, r4 = r2 * r2, r6 = r4 * r2;
    const float d = (1.0f + k[0] * r2 + k[1] * r4 + k[2] * r6) / (1.0f + k[3] * r2 + k[4] * r4 + k[5] * r6);
    const float x_y_ = x_ * y_;
    const float xd = x_ * d + 2.0f * k[6] * x_y_ + k[7] * (r2 + 2.0f * x_2);
    const float yd = y_ * d + 2.0f * k[7] * x_y_ + k[6] * (r2 + 2.0f * y_2);
    *px = u.fx * xd + u.cx;
    *py = u.fy * yd + u.cy;
}

__device__ __forceinline__ M23 jacobian_rt8(V3 p, const Uni& u, const float* k) {
    const float fx = u.fx, fy = u.fy, p1 = k[6], p2 = k[7];
    const float z = p.z;
    const float inv_z = 1.0f / z;
    const float inv_z2 = inv_z * inv_z;
    const float x_n = bsx_clamp(p.x * inv_z, u.lnx, u.lpx);
    const float y_n = bsx_clamp(p.y * inv_z, u.lny, u.lpy);
    const float xc = x_n * z, yc = y_n * z;
    const float r2 = x_n * x_n + y_n * y_n, r4 = r2 * r2, r6 = r4 * r2;
    const float n_poly = 1.0f + k[0] * r2 + k[1] * r4 + k[2] * r6;
    const float dn_poly = 1.0f + k[3] * r2 + k[4] * r4 + k[5] * r6;
    const float np_poly = k[0] + 2.0f * k[1] * r2 + 3.0f * k[2] * r4;
    const float dnp_poly = k[3] + 2.0f * k[4] * r2 + 3.0f * k[5] * r4;
    const float inv_dn = 1.0f / dn_poly;
    const float inv_dn2 = inv_dn * inv_dn;
    const float r_val = n_poly * inv_dn;
    const float rp_val = (np_poly * dn_poly - n_poly * dnp_poly) * inv_dn2;
    const float d00 = r_val + 2.0f * x_n * x_n * rp_val + 2.0f * p1 * y_n + 6.0f * p2 * x_n;
    const float d01 = 2.0f * x_n * y_n * rp_val + 2.0f * p1 * x_n + 2.0f * p2 * y_n;
    const float d10 = d01;
    const float d11 = r_val + 2.0f * y_n * y_n * rp_val + 6.0f * p1 * y_n + 2.0f * p2 * x_n;
    return M23{fx * d00 * inv_z, fy * d10 * inv_z, fx * d01 * inv_z, fy * d11 * inv_z,
               -fx * (d00 * xc + d01 * yc) * inv_z2, -fy * (d10 * xc + d11 * yc) * inv_z2};
}

__device__ __forceinline__ V3 vjp_rt8(V3 mc, const S3& cc, const Uni& u, S2 vcov, float vmx, float vmy,
                                      const float* k) {
    const float fx = u.fx, fy = u.fy, p1 = k[6], p2 = k[7];
    const float mx = mc.x, my = mc.y, mz = mc.z;
    const float inv_z = 1.0f / mz;
    const float mx_rz_raw = mx * inv_z, my_rz_raw = my * inv_z;
    const float mx_rz = bsx_clamp(mx_rz_raw, u.lnx, u.lpx);
    const float my_rz = bsx_clamp(my_rz_raw, u.lny, u.lpy);
    const bool in_x = mx_rz_raw <= u.lpx && mx_rz_raw >= u.lnx;
    const bool in_y = my_rz_raw <= u.lpy && my_rz_raw >= u.lny;
    const float xc = mx_rz * mz, yc = my_rz * mz;
    const float inv_z2 = inv_z * inv_z, inv_z3 = inv_z2 * inv_z;
    const float x = xc * inv_z, y = yc * inv_z;
    const float r2 = x * x + y * y, r4 = r2 * r2;
    const float n_poly = 1.0f + k[0] * r2 + k[1] * r4 + k[2] * r2 * r4;
    const float dn_poly = 1.0f + k[3] * r2 + k[4] * r4 + k[5] * r2 * r4;
    const float np_poly = k[0] + 2.0f * k[1] * r2 + 3.0f * k[2] * r4;
    const float dnp_poly = k[3] + 2.0f * k[4] * r2 + 3.0f * k[5] * r4;
    const float npp_poly = 2.0f * k[1] + 6.0f * k[2] * r2;
    const float dnpp_poly = 2.0f * k[4] + 6.0f * k[5] * r2;
    const float inv_dn = 1.0f / dn_poly;
    const float inv_dn2 = inv_dn * inv_dn, inv_dn3 = inv_dn2 * inv_dn;
    const float rr = n_poly * inv_dn;
    const float rrp = (np_poly * dn_poly - n_poly * dnp_poly) * inv_dn2;
    const float rrpp = (npp_poly * dn_poly * dn_poly - 2.0f * np_poly * dn_poly * dnp_poly -
                        n_poly * dnpp_poly * dn_poly + 2.0f * n_poly * dnp_poly * dnp_poly) *
                       inv_dn3;
    const float rx = 2.0f * x * rrp, ry = 2.0f * y * rrp;
    const float rpx = 2.0f * x * rrpp, rpy = 2.0f * y * rrpp;
    const float d00 = rr + 2.0f * x * x * rrp + 2.0f * p1 * y + 6.0f * p2 * x;
    const float d01 = 2.0f * x * y * rrp + 2.0f * p1 * x + 2.0f * p2 * y;
    const float d10 = d01;
    const float d11 = rr + 2.0f * y * y * rrp + 6.0f * p1 * y + 2.0f * p2 * x;
    const float js00 = fx * d00 * inv_z, js01 = fx * d01 * inv_z;
    const float js02 = -fx * (d00 * xc + d01 * yc) * inv_z2;
    const float js10 = fy * d10 * inv_z, js11 = fy * d11 * inv_z;
    const float js12 = -fy * (d10 * xc + d11 * yc) * inv_z2;
    // J_eff = J_surr S (the clamp routes x or y into z)
    const float je00 = in_x ? js00 : 0.0f, je10 = in_x ? js10 : 0.0f;
    const float je01 = in_y ? js01 : 0.0f, je11 = in_y ? js11 : 0.0f;
    const float je02 = (in_x ? 0.0f : mx_rz * js00) + (in_y ? 0.0f : my_rz * js01) + js02;
    const float je12 = (in_x ? 0.0f : mx_rz * js10) + (in_y ? 0.0f : my_rz * js11) + js12;
    float v_mx = je00 * vmx + je10 * vmy;
    float v_my = je01 * vmx + je11 * vmy;
    float v_mz = je02 * vmx + je12 * vmy;
    const VJRows ve = vj_rows(M23{je00, je10, je01, je11, je02, je12}, vcov, cc);
    const float vs_u0 = in_x ? ve.u0 : mx_rz * ve.u2, vs_v0 = in_x ? ve.v0 : mx_rz * ve.v2;
    const float vs_u1 = in_y ? ve.u1 : my_rz * ve.u2, vs_v1 = in_y ? ve.v1 : my_rz * ve.v2;
    const float vs_u2 = ve.u2, vs_v2 = ve.v2;
    const float dd00_dx = rx + 4.0f * x * rrp + 2.0f * x * x * rpx + 6.0f * p2;
    const float dd00_dy = ry + 2.0f * x * x * rpy + 2.0f * p1;
    const float dd01_dx = 2.0f * y * rrp + 2.0f * x * y * rpx + 2.0f * p1;
    const float dd01_dy = 2.0f * x * rrp + 2.0f * x * y * rpy + 2.0f * p2;
    const float dd10_dx = dd01_dx, dd10_dy = dd01_dy;
    const float dd11_dx = rx + 2.0f * y * y * rpx + 2.0f * p2;
    const float dd11_dy = ry + 4.0f * y * rrp + 2.0f * y * y * rpy + 6.0f * p1;
    const float dd00_dxc = dd00_dx * inv_z, dd00_dyc = dd00_dy * inv_z;
    const float dd00_dz = -(xc * dd00_dx + yc * dd00_dy) * inv_z2;
    const float dd01_dxc = dd01_dx * inv_z, dd01_dyc = dd01_dy * inv_z;
    const float dd01_dz = -(xc * dd01_dx + yc * dd01_dy) * inv_z2;
    const float dd10_dxc = dd10_dx * inv_z, dd10_dyc = dd10_dy * inv_z;
    const float dd10_dz = -(xc * dd10_dx + yc * dd10_dy) * inv_z2;
    const float dd11_dxc = dd11_dx * inv_z, dd11_dyc = dd11_dy * inv_z;
    const float dd11_dz = -(xc * dd11_dx + yc * dd11_dy) * inv_z2;
    const float djs00_dxc = fx * dd00_dxc * inv_z, djs00_dyc = fx * dd00_dyc * inv_z;
    const float djs00_dz = fx * (dd00_dz * inv_z - d00 * inv_z2);
    const float djs01_dxc = fx * dd01_dxc * inv_z, djs01_dyc = fx * dd01_dyc * inv_z;
    const float djs01_dz = fx * (dd01_dz * inv_z - d01 * inv_z2);
    const float djs10_dxc = fy * dd10_dxc * inv_z, djs10_dyc = fy * dd10_dyc * inv_z;
    const float djs10_dz = fy * (dd10_dz * inv_z - d10 * inv_z2);
    const float djs11_dxc = fy * dd11_dxc * inv_z, djs11_dyc = fy * dd11_dyc * inv_z;
    const float djs11_dz = fy * (dd11_dz * inv_z - d11 * inv_z2);
    const float djs02_dxc = -fx * (dd00_dxc * xc + d00 + dd01_dxc * yc) * inv_z2;
    const float djs02_dyc = -fx * (dd00_dyc * xc + dd01_dyc * yc + d01) * inv_z2;
    const float djs02_dz = -fx * ((dd00_dz * xc + dd01_dz * yc) * inv_z2 - 2.0f * (d00 * xc + d01 * yc) * inv_z3);
    const float djs12_dxc = -fy * (dd10_dxc * xc + d10 + dd11_dxc * yc) * inv_z2;
    const float djs12_dyc = -fy * (dd10_dyc * xc + dd11_dyc * yc + d11) * inv_z2;
    const float djs12_dz = -fy * ((dd10_dz * xc + dd11_dz * yc) * inv_z2 - 2.0f * (d10 * xc + d11 * yc) * inv_z3);
    const float c_xc = vs_u0 * djs00_dxc + vs_u1 * djs01_dxc + vs_u2 * djs02_dxc + vs_v0 * djs10_dxc +
                       vs_v1 * djs11_dxc + vs_v2 * djs12_dxc;
    const float c_yc = vs_u0 * djs00_dyc + vs_u1 * djs01_dyc + vs_u2 * djs02_dyc + vs_v0 * djs10_dyc +
                       vs_v1 * djs11_dyc + vs_v2 * djs12_dyc;
    const float c_z = vs_u0 * djs00_dz + vs_u1 * djs01_dz + vs_u2 * djs02_dz + vs_v0 * djs10_dz +
                      vs_v1 * djs11_dz + vs_v2 * djs12_dz;
    if (in_x) v_mx += c_xc;
    if (in_y) v_my += c_yc;
    v_mz += c_z;
    if (!in_x) v_mz += mx_rz * c_xc;
    if (!in_y) v_mz += my_rz * c_yc;
    return v3(v_mx, v_my, v_mz);
}

// ---- thin-prism fisheye: KB4 plus tangential and thin-prism terms -----------------
struct TpPolys {
    float nu, nv, dnu_dx, dnu_dy, dnv_dx, dnv_dy;
};
__device__ __forceinline__ TpPolys tp_polys(float x, float y, const float* k) {
    const float p1 = k[4], p2 = k[5], sx1 = k[6], sy1 = k[7];
    const float x2 = x * x, y2 = y * y, xy = x * y, r2 = x2 + y2;
    return TpPolys{2.0f * p1 * xy + p2 * (3.0f * x2 + y2) + sx1 * r2,
                   2.0f * p2 * xy + p1 * (x2 + 3.0f * y2) + sy1 * r2,
                   2.0f * (p1 * y + (3.0f * p2 + sx1) * x),
                   2.0f * (p1 * x + (p2 + sx1) * y),
                   2.0f * (p2 * y + (p1 + sy1) * x),
                   2.0f * (p2 * x + (3.0f * p1 + sy1) * y)};
}

__device__ __forceinline__ void project_tpf(V3 p, const Uni& u, const float* k, float* px, float* py) {
    float uk, vk;
    project_kb4(p, u, k, &uk, &vk);
    const float inv_z = 1.0f / p.z;
    const float inv_z2 = inv_z * inv_z;
    const TpPolys t = tp_polys(p.x, p.y, k);
    *px = uk + u.fx * t.nu * inv_z2;
    *py = vk + u.fy * t.nv * inv_z2;
}

__device__ __forceinline__ M23 jacobian_tpf(V3 p, const Uni& u, const float* k) {
    const M23 j = jacobian_kb4(p, u, k);
    const float inv_z = 1.0f / p.z;
    const float inv_z2 = inv_z * inv_z, inv_z3 = inv_z2 * inv_z;
    const TpPolys t = tp_polys(p.x, p.y, k);
    return M23{j.c0x + u.fx * t.dnu_dx * inv_z2, j.c0y + u.fy * t.dnv_dx * inv_z2,
               j.c1x + u.fx * t.dnu_dy * inv_z2, j.c1y + u.fy * t.dnv_dy * inv_z2,
               j.c2x + -2.0f * u.fx * t.nu * inv_z3, j.c2y + -2.0f * u.fy * t.nv * inv_z3};
}

__device__ __forceinline__ V3 vjp_tpf(const M23& J, V3 mc, const S3& cc, const Uni& u, S2 vcov, float vmx,
                                      float vmy, const float* k) {
    const V3 g = vjp_kb4(J, mc, cc, u, vcov, vmx, vmy, k);
    const float fx = u.fx, fy = u.fy, p1 = k[4], p2 = k[5], sx1 = k[6], sy1 = k[7];
    const float inv_z = 1.0f / mc.z;
    const float inv_z2 = inv_z * inv_z, inv_z3 = inv_z2 * inv_z, inv_z4 = inv_z2 * inv_z2;
    const TpPolys t = tp_polys(mc.x, mc.y, k);
    const float d2nu_dxx = 6.0f * p2 + 2.0f * sx1, d2nu_dyy = 2.0f * p2 + 2.0f * sx1, d2nu_dxy = 2.0f * p1;
    const float d2nv_dxx = 2.0f * p1 + 2.0f * sy1, d2nv_dyy = 6.0f * p1 + 2.0f * sy1, d2nv_dxy = 2.0f * p2;
    const float h_u_00 = d2nu_dxx * inv_z2, h_u_01 = d2nu_dxy * inv_z2, h_u_11 = d2nu_dyy * inv_z2;
    const float h_u_02 = -2.0f * t.dnu_dx * inv_z3, h_u_12 = -2.0f * t.dnu_dy * inv_z3;
    const float h_u_22 = 6.0f * t.nu * inv_z4;
    const float h_v_00 = d2nv_dxx * inv_z2, h_v_01 = d2nv_dxy * inv_z2, h_v_11 = d2nv_dyy * inv_z2;
    const float h_v_02 = -2.0f * t.dnv_dx * inv_z3, h_v_12 = -2.0f * t.dnv_dy * inv_z3;
    const float h_v_22 = 6.0f * t.nv * inv_z4;
    const VJRows vj = vj_rows(J, vcov, cc);
    const float v_mx = fx * (vj.u0 * h_u_00 + vj.u1 * h_u_01 + vj.u2 * h_u_02) +
                       fy * (vj.v0 * h_v_00 + vj.v1 * h_v_01 + vj.v2 * h_v_02);
    const float v_my = fx * (vj.u0 * h_u_01 + vj.u1 * h_u_11 + vj.u2 * h_u_12) +
                       fy * (vj.v0 * h_v_01 + vj.v1 * h_v_11 + vj.v2 * h_v_12);
    const float v_mz = fx * (vj.u0 * h_u_02 + vj.u1 * h_u_12 + vj.u2 * h_u_22) +
                       fy * (vj.v0 * h_v_02 + vj.v1 * h_v_12 + vj.v2 * h_v_22);
    return v3(g.x + v_mx, g.y + v_my, g.z + v_mz);
}

// ---- dispatch (camera_model/mod.rs:48-136) -------------------------------------------
__device__ __forceinline__ void project_mean(V3 p, const Uni& u, float* px, float* py) {
    switch (u.model) {
        case BSX_CAMERA_KANNALA_BRANDT_4: project_kb4(p, u, u.kp, px, py); break;
        case BSX_CAMERA_RADIAL_TANGENTIAL_8: project_rt8(p, u, u.kp, px, py); break;
        case BSX_CAMERA_THIN_PRISM_FISHEYE: project_tpf(p, u, u.kp, px, py); break;
        default: project_pinhole(p, u, px, py);
    }
}

__device__ __forceinline__ M23 project_jacobian(V3 p, const Uni& u) {
    switch (u.model) {
        case BSX_CAMERA_KANNALA_BRANDT_4: return jacobian_kb4(p, u, u.kp);
        case BSX_CAMERA_RADIAL_TANGENTIAL_8: return jacobian_rt8(p, u, u.kp);
        case BSX_CAMERA_THIN_PRISM_FISHEYE: return jacobian_tpf(p, u, u.kp);
        default: return pinhole_jacobian(p, u);
    }
}

}  // namespace bsx
