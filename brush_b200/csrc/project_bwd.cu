// project_bwd.cu - chain rule from screen-space gradients to splat parameters.
//
// Restates project_backwards_kernel
// (crates/brush-render-bwd/src/kernels/project_backwards.rs:19-263): conic
// VJP -> 2D covariance VJP -> projection Jacobian VJP of the camera model
// (kernels/camera_model/, camera_models.cuh) -> rotation/scale VJP, plus the SH
// coefficient VJP and the view-direction VJP into the mean (kernels/sh.rs).
// One thread per splat over all N rows; rows without gradient are written as
// zeros, so no separate zero-fill of the dense outputs is needed.
//
// Memory: a block owns R consecutive splats. Their transform and SH rows
// (contiguous in global memory) are copied into shared memory with coalesced
// loads, each thread works on its own rows there (odd row strides keep the
// per-thread accesses free of bank conflicts) with its raster-gradient row in
// registers, and the gradient rows go back to global memory with coalesced
// stores.
#include "sh.cuh"

namespace bsx {

namespace {

struct PbArgs {
    FusedAdam adam;
    GradPush push;
    const float* transforms;
    const float* sh;
    const float* raw_opac;
    const float* v_grad;  // [N,12]
    uint32_t n, coeffs;
    int mip;
    Uni u;
    float* v_transforms;
    float* v_sh;
    float* v_opac;
    float* v_refine;
};

__device__ __forceinline__ V3 s3mul(const S3& s, V3 v) {
    return vadd(vadd(vscale(v3(s.c00, s.c01, s.c02), v.x), vscale(v3(s.c01, s.c11, s.c12), v.y)),
                vscale(v3(s.c02, s.c12, s.c22), v.z));
}

// Pinhole projection VJP (pinhole.rs:58-123).
__device__ __forceinline__ V3 vjp_pinhole(const M23& J, V3 mean_c, const S3& cov_c, const Uni& u, S2 vcov,
                                          float vmx, float vmy) {
    const float mx = mean_c.x, my = mean_c.y, mz = mean_c.z;
    const float inv_z = 1.0f / mz;
    const float mxr = mx * inv_z, myr = my * inv_z;
    const float mxc = bsx_clamp(mxr, u.lnx, u.lpx), myc = bsx_clamp(myr, u.lny, u.lpy);
    const bool in_x = mxr <= u.lpx && mxr >= u.lnx;
    const bool in_y = myr <= u.lpy && myr >= u.lny;
    const float iz2 = inv_z * inv_z, iz3 = iz2 * inv_z;
    float v_mx = u.fx * inv_z * vmx;
    float v_my = u.fy * inv_z * vmy;
    float v_mz = -(u.fx * mx * vmx + u.fy * my * vmy) * iz2;
    const VJRows vj = vj_rows(J, vcov, cov_c);
    const float vj00 = vj.u0, vj11 = vj.v1, vj20 = vj.u2, vj21 = vj.v2;
    const float txv = mz * mxc, tyv = mz * myc;
    if (in_x) v_mx += -u.fx * iz2 * vj20;
    else v_mz += -u.fx * iz3 * vj20 * txv;
    if (in_y) v_my += -u.fy * iz2 * vj21;
    else v_mz += -u.fy * iz3 * vj21 * tyv;
    v_mz += -u.fx * iz2 * vj00 - u.fy * iz2 * vj11 + 2.0f * u.fx * txv * iz3 * vj20 + 2.0f * u.fy * tyv * iz3 * vj21;
    return v3(v_mx, v_my, v_mz);
}

// calculate_projection_vjp (camera_model/mod.rs:88-136)
__device__ __forceinline__ V3 projection_vjp(const M23& J, V3 mean_c, const S3& cov_c, const Uni& u, S2 vcov,
                                             float vmx, float vmy) {
    switch (u.model) {
        case BSX_CAMERA_KANNALA_BRANDT_4: return vjp_kb4(J, mean_c, cov_c, u, vcov, vmx, vmy, u.kp);
        case BSX_CAMERA_RADIAL_TANGENTIAL_8: return vjp_rt8(mean_c, cov_c, u, vcov, vmx, vmy, u.kp);
        case BSX_CAMERA_THIN_PRISM_FISHEYE: return vjp_tpf(J, mean_c, cov_c, u, vcov, vmx, vmy, u.kp);
        default: return vjp_pinhole(J, mean_c, cov_c, u, vcov, vmx, vmy);
    }
}

// Row index of element i of a staged block (i < 2^15, cols <= 80).
__device__ __forceinline__ uint32_t row_of(uint32_t i, float inv_cols) {
    return (uint32_t)(((float)i + 0.5f) * inv_cols);
}

// Copy `rows` rows of `cols` floats (contiguous in global memory) into shared
// memory rows of stride `stride`, or back. Loads are 16-byte words, B of them
// per thread issued before any is stored, when `src` is 16-byte aligned (a
// block's first row is, for the arrays this kernel is given; views at any
// offset are accepted, so it is checked), else single floats.
template <int B>
__device__ __forceinline__ void stage_in(float* dst, const float* __restrict__ src, uint32_t rows, uint32_t cols,
                                         uint32_t stride) {
    const float inv = 1.0f / (float)cols;
    const uint32_t n = rows * cols;
    const uint32_t n4 = (reinterpret_cast<uintptr_t>(src) & 15u) == 0 ? n / 4 : 0;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    for (uint32_t q0 = threadIdx.x; q0 < n4; q0 += B * blockDim.x) {
        float4 w[B];
#pragma unroll
        for (int k = 0; k < B; ++k) {
            const uint32_t q = q0 + k * blockDim.x;
            if (q < n4) w[k] = __ldg(s4 + q);
        }
#pragma unroll
        for (int k = 0; k < B; ++k) {
            const uint32_t q = q0 + k * blockDim.x;
            if (q < n4) {
                const float e[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
                uint32_t r = row_of(4 * q, inv), c = 4 * q - r * cols;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    dst[r * stride + c] = e[i];
                    if (++c == cols) {
                        c = 0;
                        ++r;
                    }
                }
            }
        }
    }
    for (uint32_t i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t r = row_of(i, inv);
        dst[r * stride + (i - r * cols)] = __ldg(src + i);
    }
}
__device__ __forceinline__ void stage_out(float* __restrict__ dst, const float* src, uint32_t rows, uint32_t cols,
                                          uint32_t stride) {
    const float inv = 1.0f / (float)cols;
    for (uint32_t i = threadIdx.x; i < rows * cols; i += blockDim.x) {
        const uint32_t r = row_of(i, inv);
        dst[i] = src[r * stride + (i - r * cols)];
    }
}

// Data-parallel push of the block's staged gradient rows [g0, g0 + rows) of
// group k: into slot `rank` of their owners. A block spans at most two owners
// (every shard has at least a block of rows, which the host checks); rows
// before the second owner's first row form one contiguous run, the rest a
// second one.
__device__ __forceinline__ void push_out(const GradPush& P, int k, const float* src, uint32_t g0, uint32_t rows,
                                         uint32_t cols, uint32_t stride) {
    const int q0 = shard_owner(P.n, g0, P.world);
    const uint32_t b1 = q0 + 1 < P.world ? shard_begin(P.n, q0 + 1, P.world) : P.n;
    const uint32_t split = min(rows, b1 - g0);
    float* d0 = P.dst[k][q0] + ((size_t)P.rank * P.slot_rows + (g0 - shard_begin(P.n, q0, P.world))) * cols;
    float* d1 = split < rows ? P.dst[k][q0 + 1] + (size_t)P.rank * P.slot_rows * cols : nullptr;
    const uint32_t n0 = split * cols, total = rows * cols;
    const float inv = 1.0f / (float)cols;
    // 16-byte stores (NVLink moves whole words far faster than single floats)
    // when both runs start 16-byte aligned and the first ends on a word
    const bool vec = ((reinterpret_cast<uintptr_t>(d0) | reinterpret_cast<uintptr_t>(d1)) & 15u) == 0 && n0 % 4 == 0;
    const uint32_t n4 = vec ? total / 4 : 0;
    for (uint32_t j = threadIdx.x; j < n4; j += blockDim.x) {
        uint32_t r = row_of(4 * j, inv), c = 4 * j - r * cols;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[i] = src[r * stride + c];
            if (++c == cols) {
                c = 0;
                ++r;
            }
        }
        const float4 w = make_float4(v[0], v[1], v[2], v[3]);
        if (4 * j < n0) reinterpret_cast<float4*>(d0)[j] = w;
        else reinterpret_cast<float4*>(d1)[j - n0 / 4] = w;
    }
    for (uint32_t i = 4 * n4 + threadIdx.x; i < total; i += blockDim.x) {
        const uint32_t r = row_of(i, inv);
        const float v = src[r * stride + (i - r * cols)];
        if (i < n0) d0[i] = v;
        else d1[i - n0] = v;
    }
}
__device__ __forceinline__ float* push_scalar(const GradPush& P, uint32_t g) {
    const int q = shard_owner(P.n, g, P.world);
    return P.dst[2][q] + (size_t)P.rank * P.slot_rows + (g - shard_begin(P.n, q, P.world));
}

template <int DEG>
struct PbShape {
    static constexpr int C3 = (DEG + 1) * (DEG + 1) * 3;
    static constexpr int R = DEG >= 4 ? 64 : 128;  // splats per block
    static constexpr int TS = 11;                  // transform row stride (odd)
    static constexpr int SS = C3 | 1;              // SH row stride (odd)
};

// AdamScaled element update, the expressions of adam.cu's adam_tile, in three
// parts: the second moment, its denominator sqrt(v * inv_bc2) + eps (computed
// once per row where the moment is per row) and the first-moment step.
__device__ __forceinline__ float adam_v(const FusedAdam& A, float g, float v_old) {
    const float one_m_b2 = 1.0f - A.b2;
    return A.first ? (g * g) * one_m_b2 : v_old * A.b2 + (g * g) * one_m_b2;
}
__device__ __forceinline__ float adam_den(const FusedAdam& A, float vv) { return sqrtf(vv * A.inv_bc2) + A.eps; }
__device__ __forceinline__ void adam_step(const FusedAdam& A, float p, float g, float m_old, float den, float sc,
                                          float* po, float* mo) {
    const float one_m_b1 = 1.0f - A.b1;
    const float mm = A.first ? g * one_m_b1 : m_old * A.b1 + g * one_m_b1;
    const float u = __fdividef(mm * A.inv_bc1, den);
    *po = p - u * sc;
    *mo = mm;
}

// Adam over the block's rows [g0, g0 + rows) of one group: flat and coalesced
// over parameters and moments; 16-byte words (B per stream and thread in
// flight) when every stream of the range is 16-byte aligned (arrays of any row
// count and views at any offset are accepted, so this is checked), else single
// floats; gradients from the staged rows (stride gs). With `reduce` the second
// moment is per row (already updated) and `s_den` holds its denominators.
template <int B>
__device__ __forceinline__ void adam_rows(const FusedAdam& A, float* __restrict__ param, float* __restrict__ m,
                                          float* __restrict__ v, const float* sg, uint32_t gs, uint32_t g0,
                                          uint32_t rows, uint32_t cols, float lr, const float* scale,
                                          bool reduce, const float* s_den) {
    const float inv = 1.0f / (float)cols;
    const size_t base = (size_t)g0 * cols;
    const bool aligned = ((reinterpret_cast<uintptr_t>(param + base) | reinterpret_cast<uintptr_t>(m + base) |
                           (reduce ? 0u : reinterpret_cast<uintptr_t>(v + base))) & 15u) == 0;
    const uint32_t n = rows * cols, n4 = aligned ? n / 4 : 0;
    float4* p4 = reinterpret_cast<float4*>(param + base);
    float4* m4 = reinterpret_cast<float4*>(m + base);
    float4* v4 = reinterpret_cast<float4*>(v + base);
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    auto elem = [&](uint32_t r, uint32_t c, float& p, float& mo, float& vo) {
        const float g = sg[r * gs + c] * A.gscale;
        const float sc = scale ? scale[c] * lr : lr;
        float den;
        if (reduce) {
            den = s_den[r];
        } else {
            vo = adam_v(A, g, vo);
            den = adam_den(A, vo);
        }
        adam_step(A, p, g, mo, den, sc, &p, &mo);
    };
    auto upd4 = [&](uint32_t q, float4 p, float4 mo, float4 vo) {
        float pe[4] = {p.x, p.y, p.z, p.w}, me[4] = {mo.x, mo.y, mo.z, mo.w}, ve[4] = {vo.x, vo.y, vo.z, vo.w};
        uint32_t r = row_of(4 * q, inv), c = 4 * q - r * cols;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            elem(r, c, pe[i], me[i], ve[i]);
            if (++c == cols) {
                c = 0;
                ++r;
            }
        }
        p4[q] = make_float4(pe[0], pe[1], pe[2], pe[3]);
        m4[q] = make_float4(me[0], me[1], me[2], me[3]);
        if (!reduce) v4[q] = make_float4(ve[0], ve[1], ve[2], ve[3]);
    };
    for (uint32_t q0 = threadIdx.x; q0 < n4; q0 += B * blockDim.x) {
        float4 pw[B], mw[B], vw[B];
#pragma unroll
        for (int k = 0; k < B; ++k) {
            const uint32_t q = q0 + k * blockDim.x;
            const bool in = q < n4;
            pw[k] = in ? p4[q] : zero;
            mw[k] = (A.first || !in) ? zero : m4[q];
            vw[k] = (reduce || A.first || !in) ? zero : v4[q];
        }
#pragma unroll
        for (int k = 0; k < B; ++k) {
            const uint32_t q = q0 + k * blockDim.x;
            if (q < n4) upd4(q, pw[k], mw[k], vw[k]);
        }
    }
    for (uint32_t e = 4 * n4 + threadIdx.x; e < n; e += blockDim.x) {
        const uint32_t r = row_of(e, inv), c = e - r * cols;
        float po = param[base + e], mo = A.first ? 0.0f : m[base + e], vo = (reduce || A.first) ? 0.0f : v[base + e];
        elem(r, c, po, mo, vo);
        param[base + e] = po;
        m[base + e] = mo;
        if (!reduce) v[base + e] = vo;
    }
}

// PINHOLE: the launch's camera is a pinhole, fixed at compile time so the
// fisheye models' code stays out of the common kernel.
// Six resident blocks per SM at 80 registers, no spills (seven fit the shared
// memory, but at 72 registers the kernel measured 9 % slower).
template <int DEG, bool PINHOLE, bool FUSE>
__global__ void __launch_bounds__(PbShape<DEG>::R, 6) project_bwd_kernel(const PbArgs a) {
    using S = PbShape<DEG>;
    constexpr int C3 = S::C3;
    __shared__ float s_t[S::R * S::TS];
    __shared__ float s_sh[S::R * S::SS];
    __shared__ float s_op[FUSE ? S::R : 1];    // opacity gradients (fused Adam)
    __shared__ float s_den[FUSE ? S::R : 1];   // SH Adam denominator per row (fused Adam)
    // With the gradient push, block b takes row block (b % world) K + b / world
    // (K = row blocks per owner, rounded up): any `world` consecutive blocks
    // write to different owners, so the peer stores spread over the launch.
    uint32_t blk = blockIdx.x;
    if (a.push.world) {
        const uint32_t nb = (a.n + S::R - 1) / S::R, per = (nb + a.push.world - 1) / a.push.world;
        blk = (blockIdx.x % a.push.world) * per + blockIdx.x / a.push.world;
        if (blk >= nb) return;
    }
    const uint32_t g0 = blk * S::R;
    const uint32_t rows = min((uint32_t)S::R, a.n - g0);
    const uint32_t r = threadIdx.x;
    // the row's scalar inputs, issued with the staged rows rather than after them
    const float raw_op = r < rows ? __ldg(a.raw_opac + g0 + r) : 0.0f;
    const float v_sh_old = (FUSE && r < rows && !a.adam.first) ? a.adam.v_sh[g0 + r] : 0.0f;
    // the row's raster gradients: three 16-byte words per thread straight into
    // registers (a warp reads 1.5 KB contiguous; no shared-memory staging)
    float rg[kGradStride];
    {
        const float4* gp = reinterpret_cast<const float4*>(a.v_grad + (size_t)(g0 + min(r, rows - 1)) * kGradStride);
        const float4 q0 = __ldg(gp), q1 = __ldg(gp + 1), q2 = __ldg(gp + 2);
        const float w[kGradStride] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w, q2.x, q2.y, q2.z, q2.w};
#pragma unroll
        for (int k = 0; k < kGradStride; ++k) rg[k] = w[k];
    }
    stage_in<2>(s_t, a.transforms + (size_t)g0 * 10, rows, 10, S::TS);
    stage_in<(S::C3 >= 48 ? 6 : 2)>(s_sh, a.sh + (size_t)g0 * C3, rows, C3, S::SS);
    __syncthreads();
    if (r < rows) {
        const uint32_t g = g0 + r;
        float* t = s_t + r * S::TS;   // transform in, transform gradient out
        float* shr = s_sh + r * S::SS;  // SH in, SH gradient out
        bool any = false;
#pragma unroll
        for (int k = 0; k < BSX_COMPACT_GRAD_LANES; ++k) any = any || rg[k] != 0.0f;
        if (!any) {
#pragma unroll
            for (int k = 0; k < 10; ++k) t[k] = 0.0f;
#pragma unroll
            for (int k = 0; k < C3; ++k) shr[k] = 0.0f;
            if (FUSE) s_op[r] = 0.0f;
            if (!FUSE || a.adam.keep_grads) *(a.push.world ? push_scalar(a.push, g) : a.v_opac + g) = 0.0f;
            a.v_refine[g] = 0.0f;
        } else {
            Uni u = a.u;
            if (PINHOLE) u.model = BSX_CAMERA_PINHOLE;
            const float vmx = rg[0], vmy = rg[1], vcx = rg[2], vcy = rg[3], vcz = rg[4];
            const V3 vcol = v3(rg[5], rg[6], rg[7]);
            const float valpha = rg[8], vref = rg[9], vdep = rg[10];
            const V3 mean = v3(t[0], t[1], t[2]);
            const V3 scl = v3(bsx_expf(t[7]), bsx_expf(t[8]), bsx_expf(t[9]));
            const Q4 qu{t[3], t[4], t[5], t[6]};
            const Q4 q = qnormalize(qu);

            // view direction + SH VJPs (read the coefficients before overwriting the row)
            const V3 uw = vsub(mean, u.cam);
            const float ulen = sqrtf(vdot(uw, uw));
            const V3 vdir = vscale(uw, 1.0f / ulen);
            const V3 vv = sh_viewdir_vjp<DEG>(shr, vdir, vcol);
            sh_coeffs_vjp<DEG>(shr, vdir, vcol);
            const float vdv = vdot(vdir, vv);
            const V3 v_mean_sh = vscale(vsub(vv, vscale(vdir, vdv)), 1.0f / ulen);

            const V3 mean_c = vadd(mmul(u.rot, mean), u.trans);
            const M3 R = quat_to_mat3(q);
            const M3 Mm = mdiag(R, scl);
            const S2 raw = calc_cov2d(scl, q, mean_c, u);
            float fc;
            const S2 cov = compensate_cov2d(raw, a.mip != 0, &fc);
            const float os = bsx_sigmoid(raw_op);
            const float vop = fc * valpha * os * (1.0f - os);
            if (FUSE) s_op[r] = vop;
            if (!FUSE || a.adam.keep_grads) *(a.push.world ? push_scalar(a.push, g) : a.v_opac + g) = vop;
            const float rc = bsx_is_finite(vref) ? vref : 0.0f;
            a.v_refine[g] = bsx_clamp(rc, 0.0f, 1.0e32f);

            const S2 ci = sym2_inverse(cov);
            const S2 vi{vcx, vcy * 0.5f, vcz};
            const float t00 = -ci.c00 * vi.c00 + -ci.c01 * vi.c01;
            const float t01 = -ci.c01 * vi.c00 + -ci.c11 * vi.c01;
            const float t10 = -ci.c00 * vi.c01 + -ci.c01 * vi.c11;
            const float t11 = -ci.c01 * vi.c01 + -ci.c11 * vi.c11;
            const S2 vcov{t00 * ci.c00 + t10 * ci.c01, t01 * ci.c00 + t11 * ci.c01, t01 * ci.c01 + t11 * ci.c11};

            const V3 mr0 = mrow(Mm, 0), mr1 = mrow(Mm, 1), mr2 = mrow(Mm, 2);
            const S3 covar{vdot(mr0, mr0), vdot(mr0, mr1), vdot(mr0, mr2),
                           vdot(mr1, mr1), vdot(mr1, mr2), vdot(mr2, mr2)};
            const V3 vr0 = mrow(u.rot, 0), vr1 = mrow(u.rot, 1), vr2 = mrow(u.rot, 2);
            const V3 sr0 = s3mul(covar, vr0), sr1 = s3mul(covar, vr1), sr2 = s3mul(covar, vr2);
            const S3 cov_c{vdot(vr0, sr0), vdot(vr0, sr1), vdot(vr0, sr2),
                           vdot(vr1, sr1), vdot(vr1, sr2), vdot(vr2, sr2)};
            const M23 J = project_jacobian(mean_c, u);
            const float jc[3][2] = {{J.c0x, J.c0y}, {J.c1x, J.c1y}, {J.c2x, J.c2y}};
            float tmp[3][2];
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                tmp[c][0] = vcov.c00 * jc[c][0] + vcov.c01 * jc[c][1];
                tmp[c][1] = vcov.c01 * jc[c][0] + vcov.c11 * jc[c][1];
            }
            const V3 pv = projection_vjp(J, mean_c, cov_c, u, vcov, vmx, vmy);
            const float v_mx = pv.x, v_my = pv.y, v_mz = pv.z;
            const V3 v_mean_c = v3(v_mx, v_my, v_mz + vdep);

            // J^T v_cov2d J (Mat2x3::transpose_congruence_sym2)
            const S3 vcc{jc[0][0] * tmp[0][0] + jc[0][1] * tmp[0][1], jc[0][0] * tmp[1][0] + jc[0][1] * tmp[1][1],
                         jc[0][0] * tmp[2][0] + jc[0][1] * tmp[2][1], jc[1][0] * tmp[1][0] + jc[1][1] * tmp[1][1],
                         jc[1][0] * tmp[2][0] + jc[1][1] * tmp[2][1], jc[2][0] * tmp[2][0] + jc[2][1] * tmp[2][1]};
            const V3 v_mean = vadd(mtmul(u.rot, v_mean_c), v_mean_sh);
            // v_M = 2 (R_view^T vcc R_view) M
            const V3 sc0 = s3mul(vcc, u.rot.c0), sc1 = s3mul(vcc, u.rot.c1), sc2 = s3mul(vcc, u.rot.c2);
            const S3 tc{vdot(u.rot.c0, sc0), vdot(u.rot.c0, sc1), vdot(u.rot.c0, sc2),
                        vdot(u.rot.c1, sc1), vdot(u.rot.c1, sc2), vdot(u.rot.c2, sc2)};
            const S3 tc2{tc.c00 * 2.0f, tc.c01 * 2.0f, tc.c02 * 2.0f, tc.c11 * 2.0f, tc.c12 * 2.0f, tc.c22 * 2.0f};
            const M3 vM{s3mul(tc2, Mm.c0), s3mul(tc2, Mm.c1), s3mul(tc2, Mm.c2)};
            const V3 vse = v3(vdot(R.c0, vM.c0) * scl.x, vdot(R.c1, vM.c1) * scl.y, vdot(R.c2, vM.c2) * scl.z);
            // quat_to_mat_vjp of v_M diag(scale)
            const M3 vr = mdiag(vM, scl);
            const float qw = q.w, qx = q.x, qy = q.y, qz = q.z;
            const float wg = qx * (vr.c1.z - vr.c2.y) + qy * (vr.c2.x - vr.c0.z) + qz * (vr.c0.y - vr.c1.x);
            const float xg = -2.0f * qx * (vr.c1.y + vr.c2.z) + qy * (vr.c0.y + vr.c1.x) + qz * (vr.c0.z + vr.c2.x) +
                             qw * (vr.c1.z - vr.c2.y);
            const float yg = qx * (vr.c0.y + vr.c1.x) - 2.0f * qy * (vr.c0.x + vr.c2.z) + qz * (vr.c1.z + vr.c2.y) +
                             qw * (vr.c2.x - vr.c0.z);
            const float zg = qx * (vr.c0.z + vr.c2.x) + qy * (vr.c1.z + vr.c2.y) - 2.0f * qz * (vr.c0.x + vr.c1.y) +
                             qw * (vr.c0.y - vr.c1.x);
            const Q4 qg{2.0f * wg, 2.0f * xg, 2.0f * yg, 2.0f * zg};
            // normalisation VJP on the raw quaternion
            const float lsq = qdot(qu, qu);
            const float l = sqrtf(lsq);
            const float inv = 1.0f / (l * lsq);
            const float cc0 = -qu.w * qu.x, cc1 = -qu.x * qu.y, cc2 = -qu.y * qu.w;
            const float cs0 = -qu.w * qu.z, cs1 = -qu.x * qu.z, cs2 = -qu.y * qu.z;
            const float sw_ = qu.w * qu.w, sx_ = qu.x * qu.x, sy_ = qu.y * qu.y, sz_ = qu.z * qu.z;
            t[0] = v_mean.x;
            t[1] = v_mean.y;
            t[2] = v_mean.z;
            t[3] = ((lsq - sw_) * qg.w + cc0 * qg.x + cc2 * qg.y + cs0 * qg.z) * inv;
            t[4] = (cc0 * qg.w + (lsq - sx_) * qg.x + cc1 * qg.y + cs1 * qg.z) * inv;
            t[5] = (cc2 * qg.w + cc1 * qg.x + (lsq - sy_) * qg.y + cs2 * qg.z) * inv;
            t[6] = (cs0 * qg.w + cs1 * qg.x + cs2 * qg.y + (lsq - sz_) * qg.z) * inv;
            t[7] = vse.x;
            t[8] = vse.y;
            t[9] = vse.z;
        }
    }
    __syncthreads();
    if (!FUSE && a.push.world) {
        push_out(a.push, 0, s_t, g0, rows, 10, S::TS);
        push_out(a.push, 1, s_sh, g0, rows, C3, S::SS);
        // the peer stores are made visible before the exchange kernel's release
        __threadfence_system();
    } else if (!FUSE || a.adam.keep_grads) {
        stage_out(a.v_transforms + (size_t)g0 * 10, s_t, rows, 10, S::TS);
        stage_out(a.v_sh + (size_t)g0 * C3, s_sh, rows, C3, S::SS);
    }
    if (FUSE) {
        const FusedAdam& A = a.adam;
        // SH rows: second moment from the mean square of the row (reduce_moment_2),
        // summed in adam.cu's fixed order (quads of the row in column order)
        if (r < rows) {
            const float* gr = s_sh + r * S::SS;
            float s2 = 0.0f;
            if (C3 % 4 == 0) {
                for (int i = 0; i < C3 / 4; ++i) {
                    const float x = gr[4 * i] * A.gscale, y = gr[4 * i + 1] * A.gscale, z = gr[4 * i + 2] * A.gscale,
                                w = gr[4 * i + 3] * A.gscale;
                    s2 += x * x + y * y + z * z + w * w;
                }
            } else {
                for (int c = 0; c < C3; ++c) {
                    const float gg = gr[c] * A.gscale;
                    s2 += gg * gg;
                }
            }
            const float gsq = s2 * (1.0f / (float)C3);
            const uint32_t row = g0 + r;
            const float vr = A.first ? gsq * (1.0f - A.b2) : v_sh_old * A.b2 + gsq * (1.0f - A.b2);
            A.v_sh[row] = vr;
            s_den[r] = adam_den(A, vr);
        }
        __syncthreads();
        adam_rows<3>(A, const_cast<float*>(a.transforms), A.m_t, A.v_t, s_t, S::TS, g0, rows, 10, A.lr_t,
                     A.has_t_scale ? A.t_scale : nullptr, false, nullptr);
        adam_rows<4>(A, const_cast<float*>(a.sh), A.m_sh, A.v_sh, s_sh, S::SS, g0, rows, C3, A.lr_sh,
                     A.has_sh_scale ? A.sh_scale : nullptr, true, s_den);
        adam_rows<1>(A, const_cast<float*>(a.raw_opac), A.m_o, A.v_o, s_op, 1, g0, rows, 1, A.lr_op, nullptr, false,
                     nullptr);
    }
}

template <int DEG, bool FUSE>
void launch_deg(const PbArgs& a, cudaStream_t st) {
    constexpr int R = PbShape<DEG>::R;
    uint32_t grid = (a.n + R - 1) / R;
    if (a.push.world) grid = (grid + a.push.world - 1) / a.push.world * a.push.world;  // whole rounds of owners
    if (a.u.model == BSX_CAMERA_PINHOLE) project_bwd_kernel<DEG, true, FUSE><<<grid, R, 0, st>>>(a);
    else project_bwd_kernel<DEG, false, FUSE><<<grid, R, 0, st>>>(a);
}

}  // namespace

bsx_status launch_project_bwd(bsx_ctx* ctx, const bsx_project_uniforms& uni, const float* transforms, const float* sh,
                              const float* raw_opac, uint32_t n, uint32_t coeffs, int degree, int mip,
                              const float* v_grad, float* v_transforms, float* v_sh, float* v_opac, float* v_refine,
                              const FusedAdam* adam, const GradPush* push) {
    if (n == 0) return BSX_OK;
    PbArgs a;
    if (adam) a.adam = *adam;
    a.push.world = 0;
    if (push && push->world > 1) {
        if (adam) return fail(ctx, BSX_ERR_INVALID_ARG, "gradient push and fused Adam are exclusive");
        a.push = *push;
    }
    a.transforms = transforms;
    a.sh = sh;
    a.raw_opac = raw_opac;
    a.v_grad = v_grad;
    a.n = n;
    a.coeffs = coeffs;
    a.mip = mip;
    a.u = make_uni(uni);
    a.v_transforms = v_transforms;
    a.v_sh = v_sh;
    a.v_opac = v_opac;
    a.v_refine = v_refine;
    if (degree < 0 || degree > 4) return fail(ctx, BSX_ERR_SHAPE, "unsupported SH degree");
    prof_begin(ctx);
    if (adam) {
        switch (degree) {
            case 0: launch_deg<0, true>(a, ctx->stream); break;
            case 1: launch_deg<1, true>(a, ctx->stream); break;
            case 2: launch_deg<2, true>(a, ctx->stream); break;
            case 3: launch_deg<3, true>(a, ctx->stream); break;
            default: launch_deg<4, true>(a, ctx->stream); break;
        }
    } else {
        switch (degree) {
            case 0: launch_deg<0, false>(a, ctx->stream); break;
            case 1: launch_deg<1, false>(a, ctx->stream); break;
            case 2: launch_deg<2, false>(a, ctx->stream); break;
            case 3: launch_deg<3, false>(a, ctx->stream); break;
            default: launch_deg<4, false>(a, ctx->stream); break;
        }
    }
    return post_launch(ctx, "project_bwd_kernel");
}

}  // namespace bsx
