// adam.cu - fused AdamScaled update for every parameter group in one launch.
//
// Restates AdamScaled::step / AdaptiveMomentum::transform
// (crates/brush-train/src/adam_scaled.rs:216-383):
//   m <- b1 m + (1-b1) g            (first step: (1-b1) g)
//   v <- b2 v + (1-b2) g2           (g2 = g^2, or its row mean when reduce_moment_2)
//   p <- p - (m/(1-b1^t)) / (sqrt(v/(1-b2^t)) + eps) * lr * col_scale
// The reference runs this as ~10-15 generic elementwise/reduction kernels per
// parameter tensor; here one thread owns one row of one group and does the
// whole update in registers (one read of p, g, m, v and one write of p, m, v).
#include <vector>

#include "common.cuh"

namespace bsx {

namespace {

constexpr int kAdamThreads = 256;
constexpr int kMaxGroups = 4;
constexpr int kMaxCols = 64;

struct AdamGroupDev {
    float* param;
    const float* grad;
    float* m;
    float* v;
    uint32_t rows, cols;
    float lr;
    int reduce;
    int has_scale;
    uint32_t block_begin;
    float scale[kMaxCols];
};

struct AdamArgs {
    AdamGroupDev g[kMaxGroups];
    int ngroups;
    float b1, b2, eps, bc1, bc2, gscale;
    int first;
};

__global__ void __launch_bounds__(kAdamThreads) adam_kernel(const __grid_constant__ AdamArgs a) {
    int k = 0;
    for (int i = 1; i < a.ngroups; ++i)
        if (blockIdx.x >= a.g[i].block_begin) k = i;
    const AdamGroupDev& G = a.g[k];
    const uint32_t row = (blockIdx.x - G.block_begin) * kAdamThreads + threadIdx.x;
    if (row >= G.rows) return;
    const size_t r0 = (size_t)row * G.cols;
    const float one_m_b1 = 1.0f - a.b1, one_m_b2 = 1.0f - a.b2;
    float vr = 0.0f;
    if (G.reduce) {
        float s = 0.0f;
        for (uint32_t c = 0; c < G.cols; ++c) {
            const float g = __ldg(G.grad + r0 + c) * a.gscale;
            s += g * g;
        }
        const float gsq = s / (float)G.cols;
        vr = a.first ? gsq * one_m_b2 : G.v[row] * a.b2 + gsq * one_m_b2;
        G.v[row] = vr;
    }
    for (uint32_t c = 0; c < G.cols; ++c) {
        const float g = __ldg(G.grad + r0 + c) * a.gscale;
        const float mm = a.first ? g * one_m_b1 : G.m[r0 + c] * a.b1 + g * one_m_b1;
        G.m[r0 + c] = mm;
        float vv;
        if (G.reduce) {
            vv = vr;
        } else {
            const float gsq = g * g;
            vv = a.first ? gsq * one_m_b2 : G.v[r0 + c] * a.b2 + gsq * one_m_b2;
            G.v[r0 + c] = vv;
        }
        const float upd = (mm / a.bc1) / (sqrtf(vv / a.bc2) + a.eps);
        const float s = G.has_scale ? G.scale[c] * G.lr : G.lr;
        G.param[r0 + c] = G.param[r0 + c] - upd * s;
    }
}

float powi_f32(float b, uint32_t e) {
    float r = 1.0f;
    for (uint32_t i = 0; i < e; ++i) r *= b;
    return r;
}

}  // namespace

}  // namespace bsx

using namespace bsx;

extern "C" bsx_status bsx_adam_step(bsx_ctx* ctx, const bsx_adam_group* groups, int32_t num_groups,
                                    const bsx_adam_cfg* cfg) {
    if (!ctx || !groups || !cfg || num_groups < 1) return BSX_ERR_INVALID_ARG;
    if (num_groups > kMaxGroups) return fail(ctx, BSX_ERR_UNSUPPORTED, "at most 4 parameter groups per call");
    if (cfg->step == 0) return fail(ctx, BSX_ERR_INVALID_ARG, "adam step counts from 1");
    cudaSetDevice(ctx->device);
    AdamArgs a;
    a.ngroups = num_groups;
    a.b1 = cfg->beta_1;
    a.b2 = cfg->beta_2;
    a.eps = cfg->epsilon;
    a.bc1 = 1.0f - powi_f32(cfg->beta_1, cfg->step);
    a.bc2 = 1.0f - powi_f32(cfg->beta_2, cfg->step);
    a.gscale = cfg->grad_scale;
    a.first = cfg->step == 1;
    uint32_t blocks = 0;
    for (int i = 0; i < num_groups; ++i) {
        const bsx_adam_group& s = groups[i];
        if (s.rows && (!s.d_param || !s.d_grad || !s.d_m || !s.d_v)) return fail(ctx, BSX_ERR_INVALID_ARG, "null adam buffer");
        if (s.cols == 0 || s.cols > kMaxCols) return fail(ctx, BSX_ERR_SHAPE, "adam group cols must be in [1, 64]");
        AdamGroupDev& d = a.g[i];
        d.param = s.d_param;
        d.grad = s.d_grad;
        d.m = s.d_m;
        d.v = s.d_v;
        d.rows = s.rows;
        d.cols = s.cols;
        d.lr = s.lr;
        d.reduce = s.reduce_moment_2;
        d.has_scale = s.h_col_scale != nullptr;
        for (uint32_t c = 0; c < kMaxCols; ++c) d.scale[c] = (s.h_col_scale && c < s.cols) ? s.h_col_scale[c] : 1.0f;
        d.block_begin = blocks;
        blocks += (s.rows + kAdamThreads - 1) / kAdamThreads;
    }
    if (blocks == 0) return BSX_OK;
    prof_begin(ctx);
    adam_kernel<<<blocks, kAdamThreads, 0, ctx->stream>>>(a);
    return post_launch(ctx, "adam_kernel");
}
