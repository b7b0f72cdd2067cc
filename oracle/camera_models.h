// camera_models.h - CPU restatement of the non-pinhole camera models (test oracle).
//
// TEST INFRASTRUCTURE ONLY. Included by oracle.cpp after its vector types.
// Follows crates/brush-render/src/kernels/camera_model/: kannala_brandt_4.rs
// (project :18-52, Jacobian :56-150, VJP :152-337), radial_tangential_8.rs
// (project :22-64, Jacobian :66-147, VJP :149-377) and thin_prism_fisheye.rs
// (polynomials :36-59, project :61-78, Jacobian :80-113, VJP :121-203), each
// expression in the reference's order (compiled with -ffp-contract=off); atan2
// is the shared bsx_atan2f.
#pragma once

namespace cam {

struct Intr {
    float fx, fy, cx, cy;
    float lpx, lpy, lnx, lny;
    const float* k;
};

// Rows (u0 u1 u2 v0 v1 v2) of 2 (v_cov2d J) cov_c: Sym2::mul_mat2x3 then row dots.
inline void vj_rows(const M23& J, S2 vc, const S3& cc, float out[6]) {
    float t[3][2];
    for (int c = 0; c < 3; ++c) {
        t[c][0] = vc.c00 * J.c[c][0] + vc.c01 * J.c[c][1];
        t[c][1] = vc.c01 * J.c[c][0] + vc.c11 * J.c[c][1];
    }
    V3 r0 = v3(t[0][0], t[1][0], t[2][0]), r1 = v3(t[0][1], t[1][1], t[2][1]);
    V3 c0 = v3(cc.c00, cc.c01, cc.c02), c1 = v3(cc.c01, cc.c11, cc.c12), c2 = v3(cc.c02, cc.c12, cc.c22);
    out[0] = 2.0f * dot(r0, c0);
    out[1] = 2.0f * dot(r0, c1);
    out[2] = 2.0f * dot(r0, c2);
    out[3] = 2.0f * dot(r1, c0);
    out[4] = 2.0f * dot(r1, c1);
    out[5] = 2.0f * dot(r1, c2);
}

inline M23 make_m23(float c0x, float c0y, float c1x, float c1y, float c2x, float c2y) {
    M23 m;
    m.c[0][0] = c0x; m.c[0][1] = c0y;
    m.c[1][0] = c1x; m.c[1][1] = c1y;
    m.c[2][0] = c2x; m.c[2][1] = c2y;
    return m;
}

// ---------------------------------------------------------------- KB4
inline void kb4_project(V3 p, const Intr& in, float* u, float* v) {
    float x = p.x, y = p.y, z = p.z;
    const float* k = in.k;
    float inv_z = 1.0f / z;
    float pinhole_u = in.fx * x * inv_z + in.cx;
    float pinhole_v = in.fy * y * inv_z + in.cy;
    float r = std::sqrt(x * x + y * y);
    float theta = bsx_atan2f(r, z);
    float theta2 = theta * theta;
    float theta4 = theta2 * theta2;
    float theta6 = theta2 * theta4;
    float theta8 = theta4 * theta4;
    float d = theta * (1.0f + k[0] * theta2 + k[1] * theta4 + k[2] * theta6 + k[3] * theta8);
    float inv_r = 1.0f / r;
    float fisheye_u = in.fx * (d * x * inv_r) + in.cx;
    float fisheye_v = in.fy * (d * y * inv_r) + in.cy;
    bool near_axis = r < 1e-6f;
    *u = near_axis ? pinhole_u : fisheye_u;
    *v = near_axis ? pinhole_v : fisheye_v;
}

inline M23 kb4_jacobian(V3 p, const Intr& in) {
    const float* k = in.k;
    float fx = in.fx, fy = in.fy;
    float x = p.x, y = p.y, z = p.z;
    float inv_z = 1.0f / z;
    float x2 = x * x;
    float y2 = y * y;
    float xy = x * y;
    float r2 = x2 + y2;
    float r = std::sqrt(r2);
    float inv_r = 1.0f / r;
    float inv_r3 = inv_r * inv_r * inv_r;
    float rho2 = r2 + z * z;
    float inv_rho2 = 1.0f / rho2;
    float inv_rho2_r = inv_rho2 * inv_r;
    float theta = bsx_atan2f(r, z);
    float theta2 = theta * theta;
    float theta4 = theta2 * theta2;
    float theta6 = theta4 * theta2;
    float theta8 = theta4 * theta4;
    float d = theta * (1.0f + k[0] * theta2 + k[1] * theta4 + k[2] * theta6 + k[3] * theta8);
    float dd_dtheta = 1.0f + 3.0f * k[0] * theta2 + 5.0f * k[1] * theta4 + 7.0f * k[2] * theta6 + 9.0f * k[3] * theta8;
    float dth_dx = x * z * inv_rho2_r;
    float dth_dy = y * z * inv_rho2_r;
    float dth_dz = -r * inv_rho2;
    float dd_dx = dd_dtheta * dth_dx;
    float dd_dy = dd_dtheta * dth_dy;
    float dd_dz = dd_dtheta * dth_dz;
    float xr = x * inv_r;
    float dxr_dx = y2 * inv_r3;
    float dxr_dy = -xy * inv_r3;
    float du_dx = fx * (dd_dx * xr + d * dxr_dx);
    float du_dy = fx * (dd_dy * xr + d * dxr_dy);
    float du_dz = fx * (dd_dz * xr);
    float yr = y * inv_r;
    float dyr_dx = -xy * inv_r3;
    float dyr_dy = x2 * inv_r3;
    float dv_dx = fy * (dd_dx * yr + d * dyr_dx);
    float dv_dy = fy * (dd_dy * yr + d * dyr_dy);
    float dv_dz = fy * (dd_dz * yr);
    bool near_axis = r < 1e-6f;
    float dx = fx * inv_z;
    float dy = fy * inv_z;
    float pinhole_du_dz = -dx * x * inv_z;
    float pinhole_dv_dz = -dy * y * inv_z;
    return make_m23(near_axis ? dx : du_dx, near_axis ? 0.0f : dv_dx, near_axis ? 0.0f : du_dy,
                    near_axis ? dy : dv_dy, near_axis ? pinhole_du_dz : du_dz, near_axis ? pinhole_dv_dz : dv_dz);
}

inline V3 kb4_vjp(const M23& J, V3 mean_c, const S3& cov_c, const Intr& in, S2 v_cov2d, float vmx, float vmy) {
    const float* k = in.k;
    float fx = in.fx, fy = in.fy;
    float mx = mean_c.x, my = mean_c.y, mz = mean_c.z;
    float r2 = mx * mx + my * my;
    float r = bsx_max(std::sqrt(r2), 1.0e-8f);
    float rho2 = r2 + mz * mz;
    float theta = bsx_atan2f(r, mz);
    float th2 = theta * theta;
    float th4 = th2 * th2;
    float th6 = th4 * th2;
    float th8 = th4 * th4;
    float theta_d = theta * (1.0f + k[0] * th2 + k[1] * th4 + k[2] * th6 + k[3] * th8);
    float p1 = 1.0f + 3.0f * k[0] * th2 + 5.0f * k[1] * th4 + 7.0f * k[2] * th6 + 9.0f * k[3] * th8;
    float p2 = 6.0f * k[0] * theta + 20.0f * k[1] * theta * th2 + 42.0f * k[2] * theta * th4 + 72.0f * k[3] * theta * th6;
    float inv_r = 1.0f / r;
    float inv_r3 = inv_r * inv_r * inv_r;
    float inv_r5 = inv_r3 * inv_r * inv_r;
    float inv_rho2 = 1.0f / rho2;
    float inv_rho2_sq = inv_rho2 * inv_rho2;
    float inv_rho2_r = inv_rho2 * inv_r;
    float dth_x = mx * mz * inv_rho2_r;
    float dth_y = my * mz * inv_rho2_r;
    float dth_z = -r * inv_rho2;
    float xr = mx * inv_r;
    float yr = my * inv_r;
    float dxr_x = my * my * inv_r3;
    float dxr_y = -mx * my * inv_r3;
    float dyr_x = dxr_y;
    float dyr_y = mx * mx * inv_r3;
    float dg_x = p1 * dth_x;
    float dg_y = p1 * dth_y;
    float dg_z = p1 * dth_z;
    float v_mx = vmx * J.c[0][0] + vmy * J.c[0][1];
    float v_my = vmx * J.c[1][0] + vmy * J.c[1][1];
    float v_mz = vmx * J.c[2][0] + vmy * J.c[2][1];
    float vj[6];
    vj_rows(J, v_cov2d, cov_c, vj);
    float vj_u0 = vj[0], vj_u1 = vj[1], vj_u2 = vj[2], vj_v0 = vj[3], vj_v1 = vj[4], vj_v2 = vj[5];
    float three_r2_z2 = 3.0f * r2 + mz * mz;
    float r2_minus_z2 = r2 - mz * mz;
    float h_th_00 = mz * (r2 * rho2 - mx * mx * three_r2_z2) * inv_r3 * inv_rho2_sq;
    float h_th_11 = mz * (r2 * rho2 - my * my * three_r2_z2) * inv_r3 * inv_rho2_sq;
    float h_th_01 = -mx * my * mz * three_r2_z2 * inv_r3 * inv_rho2_sq;
    float h_th_02 = mx * r2_minus_z2 * inv_r * inv_rho2_sq;
    float h_th_12 = my * r2_minus_z2 * inv_r * inv_rho2_sq;
    float h_th_22 = 2.0f * mz * r * inv_rho2_sq;
    float two_x2_my2 = 2.0f * mx * mx - my * my;
    float two_y2_mx2 = 2.0f * my * my - mx * mx;
    float h_xr_00 = -3.0f * mx * my * my * inv_r5;
    float h_xr_01 = my * two_x2_my2 * inv_r5;
    float h_xr_11 = mx * two_y2_mx2 * inv_r5;
    float h_yr_00 = my * two_x2_my2 * inv_r5;
    float h_yr_01 = mx * two_y2_mx2 * inv_r5;
    float h_yr_11 = -3.0f * mx * mx * my * inv_r5;
    float d2g, d_ju, d_jv;
    // k = 0
    d2g = p2 * dth_x * dth_x + p1 * h_th_00;
    d_ju = fx * (d2g * xr + dg_x * dxr_x + dg_x * dxr_x + theta_d * h_xr_00);
    d_jv = fy * (d2g * yr + dg_x * dyr_x + dg_x * dyr_x + theta_d * h_yr_00);
    v_mx += vj_u0 * d_ju + vj_v0 * d_jv;
    d2g = p2 * dth_y * dth_x + p1 * h_th_01;
    d_ju = fx * (d2g * xr + dg_y * dxr_x + dg_x * dxr_y + theta_d * h_xr_01);
    d_jv = fy * (d2g * yr + dg_y * dyr_x + dg_x * dyr_y + theta_d * h_yr_01);
    v_mx += vj_u1 * d_ju + vj_v1 * d_jv;
    d2g = p2 * dth_z * dth_x + p1 * h_th_02;
    d_ju = fx * (d2g * xr + dg_x * 0.0f + dg_z * dxr_x);
    d_jv = fy * (d2g * yr + dg_x * 0.0f + dg_z * dyr_x);
    v_mx += vj_u2 * d_ju + vj_v2 * d_jv;
    // k = 1
    d2g = p2 * dth_x * dth_y + p1 * h_th_01;
    d_ju = fx * (d2g * xr + dg_x * dxr_y + dg_y * dxr_x + theta_d * h_xr_01);
    d_jv = fy * (d2g * yr + dg_x * dyr_y + dg_y * dyr_x + theta_d * h_yr_01);
    v_my += vj_u0 * d_ju + vj_v0 * d_jv;
    d2g = p2 * dth_y * dth_y + p1 * h_th_11;
    d_ju = fx * (d2g * xr + dg_y * dxr_y + dg_y * dxr_y + theta_d * h_xr_11);
    d_jv = fy * (d2g * yr + dg_y * dyr_y + dg_y * dyr_y + theta_d * h_yr_11);
    v_my += vj_u1 * d_ju + vj_v1 * d_jv;
    d2g = p2 * dth_z * dth_y + p1 * h_th_12;
    d_ju = fx * (d2g * xr + dg_y * 0.0f + dg_z * dxr_y);
    d_jv = fy * (d2g * yr + dg_y * 0.0f + dg_z * dyr_y);
    v_my += vj_u2 * d_ju + vj_v2 * d_jv;
    // k = 2
    d2g = p2 * dth_x * dth_z + p1 * h_th_02;
    d_ju = fx * (d2g * xr + dg_z * dxr_x + dg_x * 0.0f);
    d_jv = fy * (d2g * yr + dg_z * dyr_x + dg_x * 0.0f);
    v_mz += vj_u0 * d_ju + vj_v0 * d_jv;
    d2g = p2 * dth_y * dth_z + p1 * h_th_12;
    d_ju = fx * (d2g * xr + dg_z * dxr_y + dg_y * 0.0f);
    d_jv = fy * (d2g * yr + dg_z * dyr_y + dg_y * 0.0f);
    v_mz += vj_u1 * d_ju + vj_v1 * d_jv;
    d2g = p2 * dth_z * dth_z + p1 * h_th_22;
    d_ju = fx * (d2g * xr);
    d_jv = fy * (d2g * yr);
    v_mz += vj_u2 * d_ju + vj_v2 * d_jv;
    return v3(v_mx, v_my, v_mz);
}

// ---------------------------------------------------------------- RT8
inline void rt8_project(V3 p, const Intr& in, float* u, float* v) {
    const float* k = in.k;
    float k1 = k[0], k2 = k[1], k3 = k[2], k4 = k[3], k5 = k[4], k6 = k[5], p1 = k[6], p2 = k[7];
    float x_ = p.x / p.z;
    float y_ = p.y / p.z;
    float x_2 = x_ * x_;
    float y_2 = y_ * y_;
    float r2 = x_2 + y_2;
    float r4 = r2 * r2;
    float r6 = r4 * r2;
    float d = (1.0f + k1 * r2 + k2 * r4 + k3 * r6) / (1.0f + k4 * r2 + k5 * r4 + k6 * r6);
    float x_y_ = x_ * y_;
    float x__ = x_ * d + 2.0f * p1 * x_y_ + p2 * (r2 + 2.0f * x_2);
    float y__ = y_ * d + 2.0f * p2 * x_y_ + p1 * (r2 + 2.0f * y_2);
    *u = in.fx * x__ + in.cx;
    *v = in.fy * y__ + in.cy;
}

inline M23 rt8_jacobian(V3 p, const Intr& in) {
    const float* k = in.k;
    float k1 = k[0], k2 = k[1], k3 = k[2], k4 = k[3], k5 = k[4], k6 = k[5], p1 = k[6], p2 = k[7];
    float fx = in.fx, fy = in.fy;
    float x = p.x, y = p.y, z = p.z;
    float inv_z = 1.0f / z;
    float inv_z2 = inv_z * inv_z;
    float x_n = bsx_clamp(x * inv_z, in.lnx, in.lpx);
    float y_n = bsx_clamp(y * inv_z, in.lny, in.lpy);
    float xc = x_n * z;
    float yc = y_n * z;
    float r2 = x_n * x_n + y_n * y_n;
    float r4 = r2 * r2;
    float r6 = r4 * r2;
    float n_poly = 1.0f + k1 * r2 + k2 * r4 + k3 * r6;
    float dn_poly = 1.0f + k4 * r2 + k5 * r4 + k6 * r6;
    float np_poly = k1 + 2.0f * k2 * r2 + 3.0f * k3 * r4;
    float dnp_poly = k4 + 2.0f * k5 * r2 + 3.0f * k6 * r4;
    float inv_dn = 1.0f / dn_poly;
    float inv_dn2 = inv_dn * inv_dn;
    float r_val = n_poly * inv_dn;
    float rp_val = (np_poly * dn_poly - n_poly * dnp_poly) * inv_dn2;
    float d00 = r_val + 2.0f * x_n * x_n * rp_val + 2.0f * p1 * y_n + 6.0f * p2 * x_n;
    float d01 = 2.0f * x_n * y_n * rp_val + 2.0f * p1 * x_n + 2.0f * p2 * y_n;
    float d10 = d01;
    float d11 = r_val + 2.0f * y_n * y_n * rp_val + 6.0f * p1 * y_n + 2.0f * p2 * x_n;
    float du_dx = fx * d00 * inv_z;
    float du_dy = fx * d01 * inv_z;
    float du_dz = -fx * (d00 * xc + d01 * yc) * inv_z2;
    float dv_dx = fy * d10 * inv_z;
    float dv_dy = fy * d11 * inv_z;
    float dv_dz = -fy * (d10 * xc + d11 * yc) * inv_z2;
    return make_m23(du_dx, dv_dx, du_dy, dv_dy, du_dz, dv_dz);
}

inline V3 rt8_vjp(V3 mean_c, const S3& cov_c, const Intr& in, S2 v_cov2d, float vmx, float vmy) {
    const float* k = in.k;
    float k1 = k[0], k2 = k[1], k3 = k[2], k4 = k[3], k5 = k[4], k6 = k[5], p1 = k[6], p2 = k[7];
    float fx = in.fx, fy = in.fy;
    float mx = mean_c.x, my = mean_c.y, mz = mean_c.z;
    float inv_z = 1.0f / mz;
    float mx_rz_raw = mx * inv_z;
    float my_rz_raw = my * inv_z;
    float mx_rz = bsx_clamp(mx_rz_raw, in.lnx, in.lpx);
    float my_rz = bsx_clamp(my_rz_raw, in.lny, in.lpy);
    bool in_x = mx_rz_raw <= in.lpx && mx_rz_raw >= in.lnx;
    bool in_y = my_rz_raw <= in.lpy && my_rz_raw >= in.lny;
    float xc = mx_rz * mz;
    float yc = my_rz * mz;
    float inv_z2 = inv_z * inv_z;
    float inv_z3 = inv_z2 * inv_z;
    float x = xc * inv_z;
    float y = yc * inv_z;
    float r2 = x * x + y * y;
    float r4 = r2 * r2;
    float n_poly = 1.0f + k1 * r2 + k2 * r4 + k3 * r2 * r4;
    float dn_poly = 1.0f + k4 * r2 + k5 * r4 + k6 * r2 * r4;
    float np_poly = k1 + 2.0f * k2 * r2 + 3.0f * k3 * r4;
    float dnp_poly = k4 + 2.0f * k5 * r2 + 3.0f * k6 * r4;
    float npp_poly = 2.0f * k2 + 6.0f * k3 * r2;
    float dnpp_poly = 2.0f * k5 + 6.0f * k6 * r2;
    float inv_dn = 1.0f / dn_poly;
    float inv_dn2 = inv_dn * inv_dn;
    float inv_dn3 = inv_dn2 * inv_dn;
    float rr = n_poly * inv_dn;
    float rrp = (np_poly * dn_poly - n_poly * dnp_poly) * inv_dn2;
    float rrpp = (npp_poly * dn_poly * dn_poly - 2.0f * np_poly * dn_poly * dnp_poly - n_poly * dnpp_poly * dn_poly +
                  2.0f * n_poly * dnp_poly * dnp_poly) *
                 inv_dn3;
    float rx = 2.0f * x * rrp;
    float ry = 2.0f * y * rrp;
    float rpx = 2.0f * x * rrpp;
    float rpy = 2.0f * y * rrpp;
    float d00 = rr + 2.0f * x * x * rrp + 2.0f * p1 * y + 6.0f * p2 * x;
    float d01 = 2.0f * x * y * rrp + 2.0f * p1 * x + 2.0f * p2 * y;
    float d10 = d01;
    float d11 = rr + 2.0f * y * y * rrp + 6.0f * p1 * y + 2.0f * p2 * x;
    float js00 = fx * d00 * inv_z;
    float js01 = fx * d01 * inv_z;
    float js02 = -fx * (d00 * xc + d01 * yc) * inv_z2;
    float js10 = fy * d10 * inv_z;
    float js11 = fy * d11 * inv_z;
    float js12 = -fy * (d10 * xc + d11 * yc) * inv_z2;
    float je00 = in_x ? js00 : 0.0f;
    float je10 = in_x ? js10 : 0.0f;
    float je01 = in_y ? js01 : 0.0f;
    float je11 = in_y ? js11 : 0.0f;
    float je02 = (in_x ? 0.0f : mx_rz * js00) + (in_y ? 0.0f : my_rz * js01) + js02;
    float je12 = (in_x ? 0.0f : mx_rz * js10) + (in_y ? 0.0f : my_rz * js11) + js12;
    float v_mx = je00 * vmx + je10 * vmy;
    float v_my = je01 * vmx + je11 * vmy;
    float v_mz = je02 * vmx + je12 * vmy;
    float ve[6];
    vj_rows(make_m23(je00, je10, je01, je11, je02, je12), v_cov2d, cov_c, ve);
    float ve_u0 = ve[0], ve_u1 = ve[1], ve_u2 = ve[2], ve_v0 = ve[3], ve_v1 = ve[4], ve_v2 = ve[5];
    float vs_u0 = in_x ? ve_u0 : mx_rz * ve_u2;
    float vs_v0 = in_x ? ve_v0 : mx_rz * ve_v2;
    float vs_u1 = in_y ? ve_u1 : my_rz * ve_u2;
    float vs_v1 = in_y ? ve_v1 : my_rz * ve_v2;
    float vs_u2 = ve_u2;
    float vs_v2 = ve_v2;
    float dd00_dx = rx + 4.0f * x * rrp + 2.0f * x * x * rpx + 6.0f * p2;
    float dd00_dy = ry + 2.0f * x * x * rpy + 2.0f * p1;
    float dd01_dx = 2.0f * y * rrp + 2.0f * x * y * rpx + 2.0f * p1;
    float dd01_dy = 2.0f * x * rrp + 2.0f * x * y * rpy + 2.0f * p2;
    float dd10_dx = dd01_dx;
    float dd10_dy = dd01_dy;
    float dd11_dx = rx + 2.0f * y * y * rpx + 2.0f * p2;
    float dd11_dy = ry + 4.0f * y * rrp + 2.0f * y * y * rpy + 6.0f * p1;
    float dd00_dxc = dd00_dx * inv_z;
    float dd00_dyc = dd00_dy * inv_z;
    float dd00_dz = -(xc * dd00_dx + yc * dd00_dy) * inv_z2;
    float dd01_dxc = dd01_dx * inv_z;
    float dd01_dyc = dd01_dy * inv_z;
    float dd01_dz = -(xc * dd01_dx + yc * dd01_dy) * inv_z2;
    float dd10_dxc = dd10_dx * inv_z;
    float dd10_dyc = dd10_dy * inv_z;
    float dd10_dz = -(xc * dd10_dx + yc * dd10_dy) * inv_z2;
    float dd11_dxc = dd11_dx * inv_z;
    float dd11_dyc = dd11_dy * inv_z;
    float dd11_dz = -(xc * dd11_dx + yc * dd11_dy) * inv_z2;
    float djs00_dxc = fx * dd00_dxc * inv_z;
    float djs00_dyc = fx * dd00_dyc * inv_z;
    float djs00_dz = fx * (dd00_dz * inv_z - d00 * inv_z2);
    float djs01_dxc = fx * dd01_dxc * inv_z;
    float djs01_dyc = fx * dd01_dyc * inv_z;
    float djs01_dz = fx * (dd01_dz * inv_z - d01 * inv_z2);
    float djs10_dxc = fy * dd10_dxc * inv_z;
    float djs10_dyc = fy * dd10_dyc * inv_z;
    float djs10_dz = fy * (dd10_dz * inv_z - d10 * inv_z2);
    float djs11_dxc = fy * dd11_dxc * inv_z;
    float djs11_dyc = fy * dd11_dyc * inv_z;
    float djs11_dz = fy * (dd11_dz * inv_z - d11 * inv_z2);
    float djs02_dxc = -fx * (dd00_dxc * xc + d00 + dd01_dxc * yc) * inv_z2;
    float djs02_dyc = -fx * (dd00_dyc * xc + dd01_dyc * yc + d01) * inv_z2;
    float djs02_dz = -fx * ((dd00_dz * xc + dd01_dz * yc) * inv_z2 - 2.0f * (d00 * xc + d01 * yc) * inv_z3);
    float djs12_dxc = -fy * (dd10_dxc * xc + d10 + dd11_dxc * yc) * inv_z2;
    float djs12_dyc = -fy * (dd10_dyc * xc + dd11_dyc * yc + d11) * inv_z2;
    float djs12_dz = -fy * ((dd10_dz * xc + dd11_dz * yc) * inv_z2 - 2.0f * (d10 * xc + d11 * yc) * inv_z3);
    float c_xc = vs_u0 * djs00_dxc + vs_u1 * djs01_dxc + vs_u2 * djs02_dxc + vs_v0 * djs10_dxc +
                 vs_v1 * djs11_dxc + vs_v2 * djs12_dxc;
    float c_yc = vs_u0 * djs00_dyc + vs_u1 * djs01_dyc + vs_u2 * djs02_dyc + vs_v0 * djs10_dyc +
                 vs_v1 * djs11_dyc + vs_v2 * djs12_dyc;
    float c_z = vs_u0 * djs00_dz + vs_u1 * djs01_dz + vs_u2 * djs02_dz + vs_v0 * djs10_dz + vs_v1 * djs11_dz +
                vs_v2 * djs12_dz;
    if (in_x) v_mx += c_xc;
    if (in_y) v_my += c_yc;
    v_mz += c_z;
    if (!in_x) v_mz += mx_rz * c_xc;
    if (!in_y) v_mz += my_rz * c_yc;
    return v3(v_mx, v_my, v_mz);
}

// ---------------------------------------------------------------- thin-prism fisheye
inline void tp_polys(float x, float y, const float* k, float out[6]) {
    float p1 = k[4], p2 = k[5], sx1 = k[6], sy1 = k[7];
    float x2 = x * x;
    float y2 = y * y;
    float xy = x * y;
    float r2 = x2 + y2;
    out[0] = 2.0f * p1 * xy + p2 * (3.0f * x2 + y2) + sx1 * r2;
    out[1] = 2.0f * p2 * xy + p1 * (x2 + 3.0f * y2) + sy1 * r2;
    out[2] = 2.0f * (p1 * y + (3.0f * p2 + sx1) * x);
    out[3] = 2.0f * (p1 * x + (p2 + sx1) * y);
    out[4] = 2.0f * (p2 * y + (p1 + sy1) * x);
    out[5] = 2.0f * (p2 * x + (3.0f * p1 + sy1) * y);
}

inline void tpf_project(V3 p, const Intr& in, float* u, float* v) {
    float uk, vk;
    kb4_project(p, in, &uk, &vk);
    float inv_z = 1.0f / p.z;
    float inv_z2 = inv_z * inv_z;
    float t[6];
    tp_polys(p.x, p.y, in.k, t);
    *u = uk + in.fx * t[0] * inv_z2;
    *v = vk + in.fy * t[1] * inv_z2;
}

inline M23 tpf_jacobian(V3 p, const Intr& in) {
    M23 j = kb4_jacobian(p, in);
    float inv_z = 1.0f / p.z;
    float inv_z2 = inv_z * inv_z;
    float inv_z3 = inv_z2 * inv_z;
    float t[6];
    tp_polys(p.x, p.y, in.k, t);
    float add_du_dx = in.fx * t[2] * inv_z2;
    float add_du_dy = in.fx * t[3] * inv_z2;
    float add_du_dz = -2.0f * in.fx * t[0] * inv_z3;
    float add_dv_dx = in.fy * t[4] * inv_z2;
    float add_dv_dy = in.fy * t[5] * inv_z2;
    float add_dv_dz = -2.0f * in.fy * t[1] * inv_z3;
    return make_m23(j.c[0][0] + add_du_dx, j.c[0][1] + add_dv_dx, j.c[1][0] + add_du_dy, j.c[1][1] + add_dv_dy,
                    j.c[2][0] + add_du_dz, j.c[2][1] + add_dv_dz);
}

inline V3 tpf_vjp(const M23& J, V3 mean_c, const S3& cov_c, const Intr& in, S2 v_cov2d, float vmx, float vmy) {
    V3 g = kb4_vjp(J, mean_c, cov_c, in, v_cov2d, vmx, vmy);
    const float* k = in.k;
    float fx = in.fx, fy = in.fy, p1 = k[4], p2 = k[5], sx1 = k[6], sy1 = k[7];
    float inv_z = 1.0f / mean_c.z;
    float inv_z2 = inv_z * inv_z;
    float inv_z3 = inv_z2 * inv_z;
    float inv_z4 = inv_z2 * inv_z2;
    float t[6];
    tp_polys(mean_c.x, mean_c.y, k, t);
    float nu = t[0], nv = t[1], dnu_dx = t[2], dnu_dy = t[3], dnv_dx = t[4], dnv_dy = t[5];
    float d2nu_dxx = 6.0f * p2 + 2.0f * sx1;
    float d2nu_dyy = 2.0f * p2 + 2.0f * sx1;
    float d2nu_dxy = 2.0f * p1;
    float d2nv_dxx = 2.0f * p1 + 2.0f * sy1;
    float d2nv_dyy = 6.0f * p1 + 2.0f * sy1;
    float d2nv_dxy = 2.0f * p2;
    float h_u_00 = d2nu_dxx * inv_z2, h_u_01 = d2nu_dxy * inv_z2, h_u_11 = d2nu_dyy * inv_z2;
    float h_u_02 = -2.0f * dnu_dx * inv_z3, h_u_12 = -2.0f * dnu_dy * inv_z3, h_u_22 = 6.0f * nu * inv_z4;
    float h_v_00 = d2nv_dxx * inv_z2, h_v_01 = d2nv_dxy * inv_z2, h_v_11 = d2nv_dyy * inv_z2;
    float h_v_02 = -2.0f * dnv_dx * inv_z3, h_v_12 = -2.0f * dnv_dy * inv_z3, h_v_22 = 6.0f * nv * inv_z4;
    float vj[6];
    vj_rows(J, v_cov2d, cov_c, vj);
    float v_mx = fx * (vj[0] * h_u_00 + vj[1] * h_u_01 + vj[2] * h_u_02) + fy * (vj[3] * h_v_00 + vj[4] * h_v_01 + vj[5] * h_v_02);
    float v_my = fx * (vj[0] * h_u_01 + vj[1] * h_u_11 + vj[2] * h_u_12) + fy * (vj[3] * h_v_01 + vj[4] * h_v_11 + vj[5] * h_v_12);
    float v_mz = fx * (vj[0] * h_u_02 + vj[1] * h_u_12 + vj[2] * h_u_22) + fy * (vj[3] * h_v_02 + vj[4] * h_v_12 + vj[5] * h_v_22);
    return v3(g.x + v_mx, g.y + v_my, g.z + v_mz);
}

}  // namespace cam
