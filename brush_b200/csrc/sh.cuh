// sh.cuh - real spherical harmonics to colour and their VJPs, degrees 0-4.
// Basis constants: Sloan, "Efficient Spherical Harmonic Evaluation", JCGT 2013,
// as used by crates/brush-render/src/kernels/sh.rs:108-555. Coefficient rows
// are [C,3] (coefficient-major, RGB-minor). Accumulation order follows the
// reference (one coefficient at a time, in index order).
#pragma once
#include "splat_math.cuh"

namespace bsx {

template <int DEG>
__device__ __forceinline__ V3 sh_to_color(const float* c, V3 v) {
    auto rc = [&](int k) { return v3(c[3 * k], c[3 * k + 1], c[3 * k + 2]); };
    V3 color = vscale(rc(0), 0.2820948f);
    if (DEG >= 1) {
        const float f0a = 0.4886025f;
        color = vadd(color, vscale(rc(1), -f0a * v.y));
        color = vadd(color, vscale(rc(2), f0a * v.z));
        color = vadd(color, vscale(rc(3), -f0a * v.x));
    }
    if (DEG >= 2) {
        float z2 = v.z * v.z;
        float f0b = -1.0925485f * v.z;
        const float f1a = 0.54627424f;
        float fc1 = v.x * v.x - v.y * v.y;
        float fs1 = 2.0f * v.x * v.y;
        float p6 = 0.9461747f * z2 - 0.31539157f;
        color = vadd(color, vscale(rc(4), f1a * fs1));
        color = vadd(color, vscale(rc(5), f0b * v.y));
        color = vadd(color, vscale(rc(6), p6));
        color = vadd(color, vscale(rc(7), f0b * v.x));
        color = vadd(color, vscale(rc(8), f1a * fc1));
        if (DEG >= 3) {
            float f0c = -2.285229f * z2 + 0.4570458f;
            float f1b = 1.4453057f * v.z;
            const float f2a = -0.5900436f;
            float fc2 = v.x * fc1 - v.y * fs1;
            float fs2 = v.x * fs1 + v.y * fc1;
            float p12 = v.z * (1.8658817f * z2 - 1.119529f);
            color = vadd(color, vscale(rc(9), f2a * fs2));
            color = vadd(color, vscale(rc(10), f1b * fs1));
            color = vadd(color, vscale(rc(11), f0c * v.y));
            color = vadd(color, vscale(rc(12), p12));
            color = vadd(color, vscale(rc(13), f0c * v.x));
            color = vadd(color, vscale(rc(14), f1b * fc1));
            color = vadd(color, vscale(rc(15), f2a * fc2));
            if (DEG >= 4) {
                float f0d = v.z * (-4.683326f * z2 + 2.0071396f);
                float f1c = 3.3116114f * z2 - 0.47308735f;
                float f2b = -1.7701308f * v.z;
                const float f3a = 0.62583575f;
                float fc3 = v.x * fc2 - v.y * fs2;
                float fs3 = v.x * fs2 + v.y * fc2;
                float p20 = 1.9843135f * v.z * p12 - 1.0062306f * p6;
                color = vadd(color, vscale(rc(16), f3a * fs3));
                color = vadd(color, vscale(rc(17), f2b * fs2));
                color = vadd(color, vscale(rc(18), f1c * fs1));
                color = vadd(color, vscale(rc(19), f0d * v.y));
                color = vadd(color, vscale(rc(20), p20));
                color = vadd(color, vscale(rc(21), f0d * v.x));
                color = vadd(color, vscale(rc(22), f1c * fc1));
                color = vadd(color, vscale(rc(23), f2b * fc2));
                color = vadd(color, vscale(rc(24), f3a * fc3));
            }
        }
    }
    return color;
}

// d colour / d coefficients, written to out[C,3] (sh.rs:476-555).
template <int DEG>
__device__ __forceinline__ void sh_coeffs_vjp(float* __restrict__ out, V3 v, V3 vc) {
    auto wc = [&](int k, float s) {
        out[3 * k] = vc.x * s;
        out[3 * k + 1] = vc.y * s;
        out[3 * k + 2] = vc.z * s;
    };
    wc(0, 0.2820948f);
    if (DEG >= 1) {
        const float f0a = 0.4886025f;
        wc(1, -f0a * v.y);
        wc(2, f0a * v.z);
        wc(3, -f0a * v.x);
    }
    if (DEG >= 2) {
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
        if (DEG >= 3) {
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
            if (DEG >= 4) {
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

// d loss / d view direction through the SH basis (sh.rs:342-470).
template <int DEG>
__device__ __forceinline__ V3 sh_viewdir_vjp(const float* c, V3 v, V3 vc) {
    auto sd = [&](int k) { return vdot(v3(c[3 * k], c[3 * k + 1], c[3 * k + 2]), vc); };
    float gx = 0.0f, gy = 0.0f, gz = 0.0f;
    if (DEG >= 1) {
        const float f0a = 0.4886025f;
        float s_n1 = sd(1), s_z0 = sd(2), s_p1 = sd(3);
        gx += -f0a * s_p1;
        gy += -f0a * s_n1;
        gz += f0a * s_z0;
    }
    if (DEG >= 2) {
        float z = v.z, x = v.x, y = v.y;
        const float c2 = -1.0925485f, f1a = 0.54627424f;
        float s_n2 = sd(4), s_n1 = sd(5), s_z0 = sd(6), s_p1 = sd(7), s_p2 = sd(8);
        gx += 2.0f * f1a * y * s_n2 + c2 * z * s_p1 + 2.0f * f1a * x * s_p2;
        gy += 2.0f * f1a * x * s_n2 + c2 * z * s_n1 - 2.0f * f1a * y * s_p2;
        gz += c2 * y * s_n1 + 2.0f * 0.9461747f * z * s_z0 + c2 * x * s_p1;
        if (DEG >= 3) {
            float z2 = z * z, x2 = x * x, y2 = y * y;
            const float f2a = -0.5900436f, c1b = 1.4453057f;
            float f1b = c1b * z;
            const float c0c = -2.285229f;
            float f0c = c0c * z2 + 0.4570458f;
            float f0c_dz = 2.0f * c0c * z;
            float s_n3 = sd(9), t_n2 = sd(10), t_n1 = sd(11), t_z0 = sd(12), t_p1 = sd(13), t_p2 = sd(14),
                  s_p3 = sd(15);
            float d12_z = 3.0f * 1.8658817f * z2 - 1.119529f;
            gx += f2a * 6.0f * x * y * s_n3 + 2.0f * f1b * y * t_n2 + f0c * t_p1 + 2.0f * f1b * x * t_p2 +
                  f2a * 3.0f * (x2 - y2) * s_p3;
            gy += f2a * 3.0f * (x2 - y2) * s_n3 + 2.0f * f1b * x * t_n2 + f0c * t_n1 + (-2.0f) * f1b * y * t_p2 +
                  f2a * (-6.0f) * x * y * s_p3;
            gz += 2.0f * c1b * x * y * t_n2 + f0c_dz * y * t_n1 + d12_z * t_z0 + f0c_dz * x * t_p1 +
                  c1b * (x2 - y2) * t_p2;
            if (DEG >= 4) {
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
                float u_n4 = sd(16), u_n3 = sd(17), u_n2 = sd(18), u_n1 = sd(19), u_z0 = sd(20), u_p1 = sd(21),
                      u_p2 = sd(22), u_p3 = sd(23), u_p4 = sd(24);
                gx += f3a * 4.0f * fs2 * u_n4 + f2b * 3.0f * fs1 * u_n3 + f1c * 2.0f * y * u_n2 + f0d * u_p1 +
                      f1c * 2.0f * x * u_p2 + f2b * 3.0f * fc1 * u_p3 + f3a * 4.0f * fc2 * u_p4;
                gy += f3a * 4.0f * fc2 * u_n4 + f2b * 3.0f * fc1 * u_n3 + f1c * 2.0f * x * u_n2 + f0d * u_n1 +
                      f1c * (-2.0f) * y * u_p2 + f2b * (-3.0f) * fs1 * u_p3 + f3a * (-4.0f) * fs2 * u_p4;
                gz += f2b_dz_const * fs2 * u_n3 + f1c_dz * fs1 * u_n2 + f0d_dz * y * u_n1 + dp_sh20_dz * u_z0 +
                      f0d_dz * x * u_p1 + f1c_dz * fc1 * u_p2 + f2b_dz_const * fc2 * u_p3;
            }
        }
    }
    return v3(gx, gy, gz);
}

}  // namespace bsx
