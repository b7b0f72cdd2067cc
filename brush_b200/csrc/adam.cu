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
constexpr int kMaxCols = 80;            // SH degree 4: 25 coefficients x 3
constexpr uint32_t kTileFloats = 4096;  // contiguous floats per block (a whole number of rows)

struct AdamGroupDev {
    float* param;
    const float* grad;
    float* m;
    float* v;
    uint32_t rows, cols, tile_rows;
    float inv_cols;
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
    float b1, b2, eps, inv_bc1, inv_bc2, gscale;
    int first;
};

// Row of element e of a tile (e < 4096, cols <= 80): the float quotient of
// e + 0.5 is never within rounding distance of an integer.
__device__ __forceinline__ uint32_t row_of(uint32_t e, float inv_cols) {
    return (uint32_t)(((float)e + 0.5f) * inv_cols);
}

// One block = one contiguous tile of whole rows of one group. The gradient
// tile is staged in shared memory with coalesced float4 loads (keeping the sum
// of squares of each float4 for reduce_moment_2 groups on the way), then p, m,
// v stream through once with coalesced float4 loads and stores. Every sum is
// taken in a fixed order, so equal inputs give bit-equal outputs on every run
// and every data-parallel replica.
__global__ void __launch_bounds__(kAdamThreads) adam_kernel(const __grid_constant__ AdamArgs a) {
    __shared__ __align__(16) float s_g[kTileFloats];
    __shared__ float s_v[kTileFloats];
    __shared__ float s_q[kTileFloats / 4];
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
    const bool vec = G.vec;
    const uint32_t nvec = vec ? count / 4 : 0;
    const bool row_quads = G.reduce && (cols % 4) == 0;  // a float4 never straddles two rows
    for (uint32_t j = threadIdx.x; j < nvec; j += kAdamThreads) {
        float4 v = __ldg(reinterpret_cast<const float4*>(G.grad + base) + j);
        v = make_float4(v.x * a.gscale, v.y * a.gscale, v.z * a.gscale, v.w * a.gscale);
        reinterpret_cast<float4*>(s_g)[j] = v;
        if (row_quads) s_q[j] = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    for (uint32_t j = nvec * 4 + threadIdx.x; j < count; j += kAdamThreads) {
        const float g = __ldg(G.grad + base + j) * a.gscale;
        s_g[j] = g;
    }
    __syncthreads();
    if (G.reduce) {
        for (uint32_t r = threadIdx.x; r < nrows; r += kAdamThreads) {
            float s2;
            if (row_quads && vec) {
                // fixed summation order: quads of the row in column order
                const uint32_t q = cols / 4;
                s2 = 0.0f;
                for (uint32_t i = 0; i < q; ++i) s2 += s_q[r * q + i];
            } else {
                s2 = 0.0f;
                for (uint32_t c = 0; c < cols; ++c) {
                    const float g = s_g[r * cols + c];
                    s2 += g * g;
                }
            }
            const float gsq = s2 * G.inv_cols;
            const float vr = a.first ? gsq * one_m_b2 : G.v[row0 + r] * a.b2 + gsq * one_m_b2;
            G.v[row0 + r] = vr;
            s_v[r] = vr;
        }
        __syncthreads();
    }
    // element update; c = column, r = row within the tile
    auto upd = [&](float p, float g, float m_old, float v_old, uint32_t c, uint32_t r, float& po, float& mo,
                   float& vo) {
        const float mm = a.first ? g * one_m_b1 : m_old * a.b1 + g * one_m_b1;
        float vv;
        if (G.reduce) {
            vv = s_v[r];
        } else {
            vv = a.first ? (g * g) * one_m_b2 : v_old * a.b2 + (g * g) * one_m_b2;
        }
        const float u = __fdividef(mm * a.inv_bc1, sqrtf(vv * a.inv_bc2) + a.eps);
        const float sc = G.has_scale ? G.scale[c] * G.lr : G.lr;
        po = p - u * sc;
        mo = mm;
        vo = vv;
    };
    if (vec) {
        float4* p4 = reinterpret_cast<float4*>(G.param + base);
        float4* m4 = reinterpret_cast<float4*>(G.m + base);
        float4* v4 = reinterpret_cast<float4*>(G.v + base);
        for (uint32_t j = threadIdx.x; j < nvec; j += kAdamThreads) {
            const uint32_t e0 = 4 * j;
            uint32_t r = row_of(e0, G.inv_cols);
            uint32_t c = e0 - r * cols;
            const float4 p = p4[j];
            const float4 g = reinterpret_cast<const float4*>(s_g)[j];
            const float4 m = a.first ? make_float4(0, 0, 0, 0) : m4[j];
            const float4 v = (G.reduce || a.first) ? make_float4(0, 0, 0, 0) : v4[j];
            float4 po, mo, vo;
            upd(p.x, g.x, m.x, v.x, c, r, po.x, mo.x, vo.x);
            if (++c == cols) { c = 0; ++r; }
            upd(p.y, g.y, m.y, v.y, c, r, po.y, mo.y, vo.y);
            if (++c == cols) { c = 0; ++r; }
            upd(p.z, g.z, m.z, v.z, c, r, po.z, mo.z, vo.z);
            if (++c == cols) { c = 0; ++r; }
            upd(p.w, g.w, m.w, v.w, c, r, po.w, mo.w, vo.w);
            p4[j] = po;
            m4[j] = mo;
            if (!G.reduce) v4[j] = vo;
        }
    }
    for (uint32_t e = nvec * 4 + threadIdx.x; e < count; e += kAdamThreads) {
        const uint32_t r = row_of(e, G.inv_cols);
        const uint32_t c = e - r * cols;
        float po, mo, vo;
        upd(G.param[base + e], s_g[e], a.first ? 0.0f : G.m[base + e], (G.reduce || a.first) ? 0.0f : G.v[base + e],
            c, r, po, mo, vo);
        G.param[base + e] = po;
        G.m[base + e] = mo;
        if (!G.reduce) G.v[base + e] = vo;
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
    a.inv_bc1 = 1.0f / (1.0f - powi_f32(cfg->beta_1, cfg->step));
    a.inv_bc2 = 1.0f / (1.0f - powi_f32(cfg->beta_2, cfg->step));
    a.gscale = cfg->grad_scale;
    a.first = cfg->step == 1;
    uint32_t blocks = 0;
    for (int i = 0; i < num_groups; ++i) {
        const bsx_adam_group& s = groups[i];
        if (s.rows && (!s.d_param || !s.d_grad || !s.d_m || !s.d_v)) return fail(ctx, BSX_ERR_INVALID_ARG, "null adam buffer");
        if (s.cols == 0 || s.cols > kMaxCols) return fail(ctx, BSX_ERR_SHAPE, "adam group cols must be in [1, 80]");
        AdamGroupDev& d = a.g[i];
        d.param = s.d_param;
        d.grad = s.d_grad;
        d.m = s.d_m;
        d.v = s.d_v;
        d.rows = s.rows;
        d.cols = s.cols;
        d.inv_cols = 1.0f / (float)s.cols;
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
