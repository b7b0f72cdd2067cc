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
constexpr uint32_t kTileFloats = 4096;  // contiguous floats per block (a whole number of rows)

struct AdamGroupDev {
    float* param;
    const float* grad;
    float* m;
    float* v;
    uint32_t rows, cols, tile_rows;
    float lr;
    int reduce;
    int has_scale;
    int vec;  // every stream 16-byte aligned and tiles a multiple of 4 floats
    uint32_t block_begin;
    float scale[kMaxCols];
};

struct AdamArgs {
    AdamGroupDev g[kMaxGroups];
    int ngroups;
    float b1, b2, eps, bc1, bc2, gscale;
    int first;
};

// One block = one contiguous tile of whole rows of one group. The gradient
// tile is staged in shared memory with coalesced (float4) loads, per-row
// second-moment means are formed there when reduce_moment_2 is set, and p, m,
// v stream through once with coalesced loads and stores.
__global__ void __launch_bounds__(kAdamThreads) adam_kernel(const __grid_constant__ AdamArgs a) {
    __shared__ __align__(16) float s_g[kTileFloats];
    __shared__ float s_v[kTileFloats];
    int k = 0;
    for (int i = 1; i < a.ngroups; ++i)
        if (blockIdx.x >= a.g[i].block_begin) k = i;
    const AdamGroupDev& G = a.g[k];
    const uint32_t row0 = (blockIdx.x - G.block_begin) * G.tile_rows;
    const uint32_t nrows = min(G.tile_rows, G.rows - row0);
    const uint32_t cols = G.cols;
    const size_t base = (size_t)row0 * cols;
    const uint32_t count = nrows * cols;
    const float one_m_b1 = 1.0f - a.b1, one_m_b2 = 1.0f - a.b2;
    if (G.vec) {
        const float4* g4 = reinterpret_cast<const float4*>(G.grad + base);
        for (uint32_t j = threadIdx.x; j < count / 4; j += kAdamThreads) {
            float4 v = __ldg(g4 + j);
            reinterpret_cast<float4*>(s_g)[j] = make_float4(v.x * a.gscale, v.y * a.gscale, v.z * a.gscale,
                                                            v.w * a.gscale);
        }
        for (uint32_t j = (count / 4) * 4 + threadIdx.x; j < count; j += kAdamThreads)
            s_g[j] = __ldg(G.grad + base + j) * a.gscale;
    } else {
        for (uint32_t j = threadIdx.x; j < count; j += kAdamThreads) s_g[j] = __ldg(G.grad + base + j) * a.gscale;
    }
    __syncthreads();
    if (G.reduce) {
        for (uint32_t r = threadIdx.x; r < nrows; r += kAdamThreads) {
            float s = 0.0f;
            for (uint32_t c = 0; c < cols; ++c) {
                const float g = s_g[r * cols + c];
                s += g * g;
            }
            const float gsq = s / (float)cols;
            const float vr = a.first ? gsq * one_m_b2 : G.v[row0 + r] * a.b2 + gsq * one_m_b2;
            G.v[row0 + r] = vr;
            s_v[r] = vr;
        }
        __syncthreads();
    }
    auto update = [&](uint32_t e, float p, float mm_old, float vv_old, float* p_out, float* m_out, float* v_out) {
        const uint32_t c = e % cols;
        const float g = s_g[e];
        const float mm = a.first ? g * one_m_b1 : mm_old * a.b1 + g * one_m_b1;
        float vv;
        if (G.reduce) {
            vv = s_v[e / cols];
        } else {
            const float gsq = g * g;
            vv = a.first ? gsq * one_m_b2 : vv_old * a.b2 + gsq * one_m_b2;
        }
        const float upd = (mm / a.bc1) / (sqrtf(vv / a.bc2) + a.eps);
        const float sc = G.has_scale ? G.scale[c] * G.lr : G.lr;
        *p_out = p - upd * sc;
        *m_out = mm;
        *v_out = vv;
    };
    if (G.vec) {
        float4* p4 = reinterpret_cast<float4*>(G.param + base);
        float4* m4 = reinterpret_cast<float4*>(G.m + base);
        float4* v4 = reinterpret_cast<float4*>(G.v + base);
        for (uint32_t j = threadIdx.x; j < count / 4; j += kAdamThreads) {
            const float4 p = p4[j];
            const float4 m = a.first ? make_float4(0, 0, 0, 0) : m4[j];
            const float4 v = (G.reduce || a.first) ? make_float4(0, 0, 0, 0) : v4[j];
            float4 po, mo, vo;
            update(4 * j + 0, p.x, m.x, v.x, &po.x, &mo.x, &vo.x);
            update(4 * j + 1, p.y, m.y, v.y, &po.y, &mo.y, &vo.y);
            update(4 * j + 2, p.z, m.z, v.z, &po.z, &mo.z, &vo.z);
            update(4 * j + 3, p.w, m.w, v.w, &po.w, &mo.w, &vo.w);
            p4[j] = po;
            m4[j] = mo;
            if (!G.reduce) v4[j] = vo;
        }
        for (uint32_t e = (count / 4) * 4 + threadIdx.x; e < count; e += kAdamThreads) {
            float po, mo, vo;
            update(e, G.param[base + e], a.first ? 0.0f : G.m[base + e],
                   (G.reduce || a.first) ? 0.0f : G.v[base + e], &po, &mo, &vo);
            G.param[base + e] = po;
            G.m[base + e] = mo;
            if (!G.reduce) G.v[base + e] = vo;
        }
    } else {
        for (uint32_t e = threadIdx.x; e < count; e += kAdamThreads) {
            float po, mo, vo;
            update(e, G.param[base + e], a.first ? 0.0f : G.m[base + e],
                   (G.reduce || a.first) ? 0.0f : G.v[base + e], &po, &mo, &vo);
            G.param[base + e] = po;
            G.m[base + e] = mo;
            if (!G.reduce) G.v[base + e] = vo;
        }
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
        // whole rows per tile, a multiple of 4 rows so every tile starts 16-byte aligned
        uint32_t tr = kTileFloats / s.cols;
        tr = tr >= 4 ? tr / 4 * 4 : tr;
        d.tile_rows = tr;
        auto al = [](const void* p) { return ((uintptr_t)p % 16) == 0; };
        d.vec = al(s.d_param) && al(s.d_grad) && al(s.d_m) && (s.reduce_moment_2 || al(s.d_v)) && (tr * s.cols) % 4 == 0;
        d.block_begin = blocks;
        blocks += (s.rows + tr - 1) / tr;
    }
    if (blocks == 0) return BSX_OK;
    prof_begin(ctx);
    adam_kernel<<<blocks, kAdamThreads, 0, ctx->stream>>>(a);
    return post_launch(ctx, "adam_kernel");
}
