// adam.cu - fused AdamScaled update for every parameter group in one launch,
// and its data-parallel form fused with the gradient exchange.
//
// Restates AdamScaled::step / AdaptiveMomentum::transform
// (crates/brush-train/src/adam_scaled.rs:216-383):
//   m <- b1 m + (1-b1) g            (first step: (1-b1) g)
//   v <- b2 v + (1-b2) g2           (g2 = g^2, or its row mean when reduce_moment_2)
//   p <- p - (m/(1-b1^t)) / (sqrt(v/(1-b2^t)) + eps) * lr * col_scale
// The reference runs this as ~10-15 generic elementwise/reduction kernels per
// parameter tensor; here one block owns one tile of whole rows of one group
// and does the whole update on chip (one read of p, g, m, v and one write of
// p, m, v).
//
// Data-parallel form (bsx_dp_adam_step): each rank owns a row shard. The
// block reads its tile's gradient from every rank's buffer (peer loads over
// NVLink, summed in rank order) or, when the ranks pushed their rows into this
// rank's gradient slots, from those local slots in the same order; updates;
// and writes the new rows into every rank's parameters (peer stores). Arrival / departure flags in each rank's
// flag words order the exchange against the ranks' neighbouring steps; every
// wait is bounded by a wall-clock timeout.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace bsx {

namespace {

constexpr int kAdamThreads = 256;
constexpr int kMaxGroups = 4;
constexpr int kMaxCols = 80;            // SH degree 4: 25 coefficients x 3
constexpr int kMaxRanks = BSX_MAX_RANKS;
constexpr uint32_t kTileFloats = 4096;  // contiguous floats per block (a whole number of rows)
// flag words: [0, 8) arrival epoch of rank q, [8, 16) departure epoch of rank q, 16 local block counter
constexpr int kFlagArrive = 0;
constexpr int kFlagDepart = 8;
constexpr int kFlagDone = 16;
static_assert(kFlagDone < BSX_DP_FLAG_WORDS, "flag layout");

struct AdamGroupDev {
    float* param;        // own parameter rows of this tile range (shard base in the data-parallel form)
    const float* grad;   // local form only
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
    float* peer_param[kMaxRanks];       // data-parallel form: every rank's shard base
    const float* peer_grad[kMaxRanks];
    float* mc_param;                    // multicast form: the shard base in the multicast mappings
    const float* mc_grad;
};

// Rows MAX-combined over the ranks in place (refine weights, noise gate).
struct MaxRows {
    float* rows[kMaxRanks];  // shard base of every rank's rows (null: none)
    float* mc;               // multicast form: shard base in the multicast mapping
    uint32_t count;          // rows of this rank's shard
    uint32_t block_begin;    // first tile of this array
    int vec;
};

struct DpDev {
    int rank, world;
    uint32_t epoch;
    uint64_t timeout_ns;
    uint32_t* flags[kMaxRanks];
    MaxRows mx[2];             // refine weights, noise gate
    uint32_t refine_block_begin;  // first MAX tile (the Adam tiles come before)
    uint32_t total_tiles;
};

struct AdamArgs {
    AdamGroupDev g[kMaxGroups];
    int ngroups;
    float b1, b2, eps, inv_bc1, inv_bc2, gscale;
    int first;
    int* err;
    DpDev dp;
};

// Row of element e of a tile (e < 4096, cols <= 80): the float quotient of
// e + 0.5 is never within rounding distance of an integer.
__device__ __forceinline__ uint32_t row_of(uint32_t e, float inv_cols) {
    return (uint32_t)(((float)e + 0.5f) * inv_cols);
}

__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4max(float4 a, float4 b) {
    return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
}

// NVLink multicast accesses (NVSwitch): a load that returns the sum (or the
// maximum) of the addressed word over every GPU bound to the multicast object,
// reduced in the switch, and a store that writes every bound GPU's copy.
__device__ __forceinline__ float4 mc_ld_add4(const float* p) {
    float4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
__device__ __forceinline__ float mc_ld_add(const float* p) {
    float r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(r) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ void mc_st4(float* p, float4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void mc_st(float* p, float v) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
// Maximum of non-negative floats as the maximum of their bit patterns.
__device__ __forceinline__ float mc_ld_max_nonneg(const float* p) {
    uint32_t r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.max.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
    return __uint_as_float(r);
}

// Waits until flags[word0 + q] has reached epoch for every rank q (threads
// 0..world-1 each poll one word). Returns false, with the error recorded,
// when the wait outlasts the timeout.
__device__ bool wait_all_ranks(const DpDev& d, int word0, int* err) {
    bool ok = true;
    if ((int)threadIdx.x < d.world) {
        const uint32_t* f = d.flags[d.rank] + word0 + threadIdx.x;
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 0;; ++it) {
            if ((int32_t)(ld_acquire_sys_u32(f) - d.epoch) >= 0) break;
            if (global_timer_ns() - t0 > d.timeout_ns || it > (1u << 28)) {
                set_error(err, kDevPeerTimeout);
                ok = false;
                break;
            }
            __nanosleep(128);
        }
    }
    return ok;
}

// Raises this rank's flag word0 + rank to epoch on every rank.
__device__ void signal_all_ranks(const DpDev& d, int word0) {
    __threadfence_system();
    if ((int)threadIdx.x < d.world) st_release_sys_u32(d.flags[threadIdx.x] + word0 + d.rank, d.epoch);
}

// MAX over ranks of one tile of this rank's shard of a combined array,
// written back to every rank.
__device__ void max_tile(const AdamArgs& a, uint32_t t) {
    const DpDev& d = a.dp;
    const MaxRows& x = d.mx[(d.mx[1].count && t >= d.mx[1].block_begin) ? 1 : 0];
    const uint32_t r0 = (t - x.block_begin) * kTileFloats;
    const uint32_t cnt = min(kTileFloats, x.count - r0);
    if (x.mc) {
        // every in-switch load of the tile in flight before the first store
        constexpr int kPer = kTileFloats / kAdamThreads;
        float v[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t e = threadIdx.x + k * kAdamThreads;
            v[k] = e < cnt ? mc_ld_max_nonneg(x.mc + r0 + e) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t e = threadIdx.x + k * kAdamThreads;
            if (e < cnt) mc_st(x.mc + r0 + e, v[k]);
        }
        return;
    }
    const uint32_t nvec = x.vec ? cnt / 4 : 0;
    for (uint32_t j = threadIdx.x; j < nvec; j += kAdamThreads) {
        float4 m = __ldcg(reinterpret_cast<const float4*>(x.rows[0] + r0) + j);
        for (int q = 1; q < d.world; ++q) m = f4max(m, __ldcg(reinterpret_cast<const float4*>(x.rows[q] + r0) + j));
        for (int q = 0; q < d.world; ++q) reinterpret_cast<float4*>(x.rows[q] + r0)[j] = m;
    }
    for (uint32_t e = nvec * 4 + threadIdx.x; e < cnt; e += kAdamThreads) {
        float m = __ldcg(x.rows[0] + r0 + e);
        for (int q = 1; q < d.world; ++q) m = fmaxf(m, __ldcg(x.rows[q] + r0 + e));
        for (int q = 0; q < d.world; ++q) x.rows[q][r0 + e] = m;
    }
}

constexpr int kVecPerThread = kTileFloats / 4 / kAdamThreads;  // float4 words per thread per tile (4)

__device__ __forceinline__ float4 ld_grad4(const float* p, uint32_t j, bool peers) {
    return peers ? __ldcg(reinterpret_cast<const float4*>(p) + j) : __ldg(reinterpret_cast<const float4*>(p) + j);
}

// One tile = a contiguous run of whole rows of one group. The gradient tile is
// staged in shared memory with coalesced float4 loads (summed over the ranks
// in rank order in the data-parallel form, and keeping the sum of squares of
// each float4 for reduce_moment_2 groups), then p, m, v stream through once
// with coalesced float4 loads and stores. Each thread owns 4 float4 words of
// the tile and issues all its loads of a phase before using them (several
// requests in flight per thread: HBM and NVLink are latency-bound otherwise).
// Every sum is taken in a fixed order, so equal inputs give bit-equal outputs
// on every run and every data-parallel replica. kW bounds the rank count.
template <bool kPeers, int kW, bool kMC = false>
__device__ void adam_tile(const AdamArgs& a, int k, uint32_t tile) {
    __shared__ __align__(16) float s_g[kTileFloats];
    __shared__ float s_v[kTileFloats];
    __shared__ float s_q[kTileFloats / 4];
    const AdamGroupDev& G = a.g[k];
    const uint32_t row0 = (tile - G.block_begin) * G.tile_rows;
    const uint32_t nrows = min(G.tile_rows, G.rows - row0);
    const uint32_t cols = G.cols;
    const size_t base = (size_t)row0 * cols;
    const uint32_t count = nrows * cols;
    const float one_m_b1 = 1.0f - a.b1, one_m_b2 = 1.0f - a.b2;
    const bool vec = G.vec;
    const uint32_t nvec = vec ? count / 4 : 0;
    const int world = kPeers ? a.dp.world : 1;
    const bool row_quads = G.reduce && (cols % 4) == 0;  // a float4 never straddles two rows
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (vec) {
        // words loaded per batch: the local form keeps one in flight per thread
        // (low registers, six resident blocks per SM measured fastest on HBM);
        // the peer form batches so that NVLink round trips overlap
        constexpr int kChunk = !kPeers ? 1 : (kW > 4 && !kMC) ? kVecPerThread / 2 : kVecPerThread;
        constexpr int kUnroll = kPeers ? kVecPerThread / kChunk : 1;
#pragma unroll kUnroll
        for (int c0 = 0; c0 < kVecPerThread; c0 += kChunk) {
            float4 acc[kChunk];
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
                const uint32_t j = threadIdx.x + (c0 + c) * kAdamThreads;
                if (kMC) acc[c] = j < nvec ? mc_ld_add4(G.mc_grad + base + 4 * (size_t)j) : zero;
                else acc[c] = j < nvec ? ld_grad4((kPeers ? G.peer_grad[0] : G.grad) + base, j, kPeers) : zero;
            }
            if (kPeers && !kMC) {
                float4 t[kW > 1 ? kW - 1 : 1][kChunk];
#pragma unroll
                for (int q = 1; q < kW; ++q)
#pragma unroll
                    for (int c = 0; c < kChunk; ++c) {
                        const uint32_t j = threadIdx.x + (c0 + c) * kAdamThreads;
                        t[q - 1][c] = (q < world && j < nvec) ? ld_grad4(G.peer_grad[q] + base, j, true) : zero;
                    }
#pragma unroll
                for (int q = 1; q < kW; ++q)
                    if (q < world)
#pragma unroll
                        for (int c = 0; c < kChunk; ++c) acc[c] = f4add(acc[c], t[q - 1][c]);
            }
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
                const uint32_t j = threadIdx.x + (c0 + c) * kAdamThreads;
                if (j < nvec) {
                    const float4 v = make_float4(acc[c].x * a.gscale, acc[c].y * a.gscale, acc[c].z * a.gscale,
                                                 acc[c].w * a.gscale);
                    reinterpret_cast<float4*>(s_g)[j] = v;
                    if (row_quads) s_q[j] = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
            }
        }
    }
    for (uint32_t j = nvec * 4 + threadIdx.x; j < count; j += kAdamThreads) {
        float g;
        if (kMC) {
            g = mc_ld_add(G.mc_grad + base + j);
        } else if (kPeers) {
            g = __ldcg(G.peer_grad[0] + base + j);
            for (int q = 1; q < world; ++q) g += __ldcg(G.peer_grad[q] + base + j);
        } else {
            g = __ldg(G.grad + base + j);
        }
        s_g[j] = g * a.gscale;
    }
    __syncthreads();
    if (G.reduce) {
        for (uint32_t r = threadIdx.x; r < nrows; r += kAdamThreads) {
            float s2 = 0.0f;
            if (row_quads && vec) {
                // fixed summation order: quads of the row in column order
                const uint32_t q = cols / 4;
                for (uint32_t i = 0; i < q; ++i) s2 += s_q[r * q + i];
            } else {
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
        constexpr int kChunkU = kPeers ? kVecPerThread : 1;
#pragma unroll 1
        for (int c0 = 0; c0 < kVecPerThread; c0 += kChunkU) {
        float4 pr[kChunkU], mr[kChunkU], vr[kChunkU];
#pragma unroll
        for (int c = 0; c < kChunkU; ++c) {
            const uint32_t j = threadIdx.x + (c0 + c) * kAdamThreads;
            const bool in = j < nvec;
            pr[c] = in ? p4[j] : zero;
            mr[c] = (in && !a.first) ? m4[j] : zero;
            vr[c] = (in && !G.reduce && !a.first) ? v4[j] : zero;
        }
#pragma unroll
        for (int c = 0; c < kChunkU; ++c) {
            const uint32_t j = threadIdx.x + (c0 + c) * kAdamThreads;
            if (j < nvec) {
                const uint32_t e0 = 4 * j;
                uint32_t r = row_of(e0, G.inv_cols);
                uint32_t col = e0 - r * cols;
                const float4 p = pr[c], m = mr[c], v = vr[c];
                const float4 g = reinterpret_cast<const float4*>(s_g)[j];
                float4 po, mo, vo;
                upd(p.x, g.x, m.x, v.x, col, r, po.x, mo.x, vo.x);
                if (++col == cols) { col = 0; ++r; }
                upd(p.y, g.y, m.y, v.y, col, r, po.y, mo.y, vo.y);
                if (++col == cols) { col = 0; ++r; }
                upd(p.z, g.z, m.z, v.z, col, r, po.z, mo.z, vo.z);
                if (++col == cols) { col = 0; ++r; }
                upd(p.w, g.w, m.w, v.w, col, r, po.w, mo.w, vo.w);
                if (kMC) mc_st4(G.mc_param + base + 4 * (size_t)j, po);  // every rank's copy, this one included
                else p4[j] = po;
                if (kPeers && !kMC)
#pragma unroll
                    for (int q = 0; q < kW; ++q)
                        if (q < world && q != a.dp.rank) reinterpret_cast<float4*>(G.peer_param[q] + base)[j] = po;
                m4[j] = mo;
                if (!G.reduce) v4[j] = vo;
            }
        }
        }
    }
    for (uint32_t e = nvec * 4 + threadIdx.x; e < count; e += kAdamThreads) {
        const uint32_t r = row_of(e, G.inv_cols);
        const uint32_t c = e - r * cols;
        float po, mo, vo;
        upd(G.param[base + e], s_g[e], a.first ? 0.0f : G.m[base + e], (G.reduce || a.first) ? 0.0f : G.v[base + e],
            c, r, po, mo, vo);
        if (kMC) mc_st(G.mc_param + base + e, po);
        else G.param[base + e] = po;
        if (kPeers && !kMC)
            for (int q = 0; q < world; ++q)
                if (q != a.dp.rank) G.peer_param[q][base + e] = po;
        G.m[base + e] = mo;
        if (!G.reduce) G.v[base + e] = vo;
    }
}

__device__ __forceinline__ int group_of(const AdamArgs& a, uint32_t tile) {
    int k = 0;
    for (int i = 1; i < a.ngroups; ++i)
        if (tile >= a.g[i].block_begin) k = i;
    return k;
}

__global__ void __launch_bounds__(kAdamThreads) adam_kernel(const __grid_constant__ AdamArgs a) {
    adam_tile<false, 1>(a, group_of(a, blockIdx.x), blockIdx.x);
}

// Data-parallel exchange + update, persistent: block b takes tiles b, b + grid,
// ...; tiles [0, refine_block_begin) are Adam tiles, the rest refine tiles.
// Every block signals its rank's arrival (idempotent) and waits for all ranks;
// the last block to finish signals departure and waits until every rank has
// departed, so the launch ends only when no rank still reads this rank's
// gradients or writes its parameters.
template <int kW, bool kMC>
__global__ void __launch_bounds__(kAdamThreads) dp_adam_kernel(const __grid_constant__ AdamArgs a) {
    const DpDev& d = a.dp;
    signal_all_ranks(d, kFlagArrive);
    const bool arrived = __syncthreads_and(wait_all_ranks(d, kFlagArrive, a.err));
    if (arrived) {
        for (uint32_t t = blockIdx.x; t < d.total_tiles; t += gridDim.x) {
            if (t < d.refine_block_begin)
                adam_tile<true, kW, kMC>(a, group_of(a, t), t);
            else
                max_tile(a, t);
            __syncthreads();  // shared staging is reused by the next tile
        }
    }
    // every thread's peer stores are ordered before the block's completion count
    __threadfence_system();
    __syncthreads();
    __shared__ uint32_t s_last;
    if (threadIdx.x == 0) {
        const uint32_t t = atomicAdd(d.flags[d.rank] + kFlagDone, 1u);
        s_last = t == gridDim.x - 1;
        if (s_last) {
            __threadfence_system();
            st_relaxed_u32(d.flags[d.rank] + kFlagDone, 0u);
        }
    }
    __syncthreads();
    if (!s_last) return;
    signal_all_ranks(d, kFlagDepart);
    wait_all_ranks(d, kFlagDepart, a.err);
}

float powi_f32(float b, uint32_t e) {
    float r = 1.0f;
    for (uint32_t i = 0; i < e; ++i) r *= b;
    return r;
}

bool aligned16(const void* p) { return ((uintptr_t)p % 16) == 0; }

// Fills the fields shared by both forms; returns the blocks the group needs.
uint32_t setup_group(AdamGroupDev& d, uint32_t rows, uint32_t cols, float lr, const float* h_scale, int reduce,
                     uint32_t block_begin) {
    d.rows = rows;
    d.cols = cols;
    d.inv_cols = 1.0f / (float)cols;
    d.lr = lr;
    d.reduce = reduce;
    d.has_scale = h_scale != nullptr;
    for (uint32_t c = 0; c < kMaxCols; ++c) d.scale[c] = (h_scale && c < cols) ? h_scale[c] : 1.0f;
    // whole rows per tile, a multiple of 4 rows so every tile starts 16-byte aligned
    uint32_t tr = kTileFloats / cols;
    tr = tr >= 4 ? tr / 4 * 4 : tr;
    d.tile_rows = tr;
    d.block_begin = block_begin;
    return (rows + tr - 1) / tr;
}

void fill_cfg(AdamArgs& a, const bsx_adam_cfg* cfg, int num_groups) {
    a.ngroups = num_groups;
    a.b1 = cfg->beta_1;
    a.b2 = cfg->beta_2;
    a.eps = cfg->epsilon;
    a.inv_bc1 = 1.0f / (1.0f - powi_f32(cfg->beta_1, cfg->step));
    a.inv_bc2 = 1.0f / (1.0f - powi_f32(cfg->beta_2, cfg->step));
    a.gscale = cfg->grad_scale;
    a.first = cfg->step == 1;
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
    fill_cfg(a, cfg, num_groups);
    a.err = ctx->d_err;
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
        const uint32_t nb = setup_group(d, s.rows, s.cols, s.lr, s.h_col_scale, s.reduce_moment_2, blocks);
        d.vec = aligned16(s.d_param) && aligned16(s.d_grad) && aligned16(s.d_m) &&
                (s.reduce_moment_2 || aligned16(s.d_v)) && (d.tile_rows * s.cols) % 4 == 0;
        blocks += nb;
    }
    if (blocks == 0) return BSX_OK;
    prof_begin(ctx);
    adam_kernel<<<blocks, kAdamThreads, 0, ctx->stream>>>(a);
    return post_launch(ctx, "adam_kernel");
}

extern "C" bsx_status bsx_dp_adam_step(bsx_ctx* ctx, const bsx_dp_exchange* ex, const bsx_dp_group* groups,
                                       int32_t num_groups, const bsx_adam_cfg* cfg) {
    if (!ctx || !ex || !groups || !cfg || num_groups < 1) return BSX_ERR_INVALID_ARG;
    if (num_groups > kMaxGroups) return fail(ctx, BSX_ERR_UNSUPPORTED, "at most 4 parameter groups per call");
    if (cfg->step == 0) return fail(ctx, BSX_ERR_INVALID_ARG, "adam step counts from 1");
    const int world = ex->world, rank = ex->rank;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(ctx, BSX_ERR_INVALID_ARG, "rank / world out of range (world <= 8)");
    if (ex->epoch == 0) return fail(ctx, BSX_ERR_INVALID_ARG, "exchange epochs count from 1");
    for (int q = 0; q < world; ++q) {
        if (!ex->d_flags[q]) return fail(ctx, BSX_ERR_INVALID_ARG, "null flag words");
        if (ex->refine_rows && !ex->d_refine[q]) return fail(ctx, BSX_ERR_INVALID_ARG, "null refine buffer");
        if (ex->gate_rows && !ex->d_gate[q]) return fail(ctx, BSX_ERR_INVALID_ARG, "null gate buffer");
    }
    cudaSetDevice(ctx->device);
    AdamArgs a;
    fill_cfg(a, cfg, num_groups);
    a.err = ctx->d_err;
    DpDev& d = a.dp;
    d.rank = rank;
    d.world = world;
    d.epoch = ex->epoch;
    d.timeout_ns = ex->timeout_ns ? ex->timeout_ns : 5000000000ull;
    auto shard = [&](uint32_t rows, uint32_t* b, uint32_t* e) {
        *b = (uint32_t)((uint64_t)rows * rank / world);
        *e = (uint32_t)((uint64_t)rows * (rank + 1) / world);
    };
    // multicast form: every group has both multicast addresses
    bool mc = true;
    for (int i = 0; i < num_groups; ++i) mc = mc && groups[i].d_param_mc && groups[i].d_grad_mc;
    if (mc && ex->grad_slot_rows) return fail(ctx, BSX_ERR_INVALID_ARG, "the multicast form reads dense gradients");
    if (mc && ((ex->refine_rows && !ex->d_refine_mc) || (ex->gate_rows && !ex->d_gate_mc)))
        return fail(ctx, BSX_ERR_INVALID_ARG, "the multicast form needs multicast refine / gate addresses");
    uint32_t blocks = 0;
    for (int i = 0; i < num_groups; ++i) {
        const bsx_dp_group& s = groups[i];
        if (s.cols == 0 || s.cols > kMaxCols) return fail(ctx, BSX_ERR_SHAPE, "adam group cols must be in [1, 80]");
        uint32_t rb, re;
        shard(s.rows, &rb, &re);
        if (re > rb && (!s.d_m || !s.d_v)) return fail(ctx, BSX_ERR_INVALID_ARG, "null adam moment buffer");
        AdamGroupDev& g = a.g[i];
        bool vec = aligned16(s.d_m) && (s.reduce_moment_2 || aligned16(s.d_v));
        for (int q = 0; q < kMaxRanks; ++q) {
            g.peer_param[q] = nullptr;
            g.peer_grad[q] = nullptr;
        }
        g.mc_param = nullptr;
        g.mc_grad = nullptr;
        if (ex->grad_slot_rows && (ex->grad_slot_rows < re - rb || !s.d_grad[rank]))
            return fail(ctx, BSX_ERR_INVALID_ARG, "gradient slots smaller than the shard");
        if (mc) {
            if (!s.d_param[rank]) return fail(ctx, BSX_ERR_INVALID_ARG, "null parameter");
            g.peer_param[rank] = s.d_param[rank] + (size_t)rb * s.cols;
            g.mc_param = s.d_param_mc + (size_t)rb * s.cols;
            g.mc_grad = s.d_grad_mc + (size_t)rb * s.cols;
            vec = vec && aligned16(g.peer_param[rank]) && aligned16(g.mc_param) && aligned16(g.mc_grad);
        }
        for (int q = 0; q < world && !mc; ++q) {
            if (!s.d_param[q] || (!ex->grad_slot_rows && !s.d_grad[q]))
                return fail(ctx, BSX_ERR_INVALID_ARG, "null parameter / gradient");
            g.peer_param[q] = s.d_param[q] + (size_t)rb * s.cols;
            // slots: rank q's rows of this shard sit in this rank's own buffer
            g.peer_grad[q] = ex->grad_slot_rows ? s.d_grad[rank] + (size_t)q * ex->grad_slot_rows * s.cols
                                                : s.d_grad[q] + (size_t)rb * s.cols;
            vec = vec && aligned16(g.peer_param[q]) && aligned16(g.peer_grad[q]);
        }
        g.param = g.peer_param[rank];
        g.grad = nullptr;
        g.m = s.d_m;
        g.v = s.d_v;
        const uint32_t nb = setup_group(g, re - rb, s.cols, s.lr, s.h_col_scale, s.reduce_moment_2, blocks);
        g.vec = vec && (g.tile_rows * s.cols) % 4 == 0;
        blocks += nb;
    }
    d.refine_block_begin = blocks;
    for (int q = 0; q < kMaxRanks; ++q) d.flags[q] = q < world ? ex->d_flags[q] : nullptr;
    float* const* srcs[2] = {ex->d_refine, ex->d_gate};
    float* const mcs[2] = {ex->d_refine_mc, ex->d_gate_mc};
    const uint32_t counts[2] = {ex->refine_rows, ex->gate_rows};
    for (int k = 0; k < 2; ++k) {
        MaxRows& x = d.mx[k];
        x.count = 0;
        x.vec = 1;
        x.block_begin = blocks;
        x.mc = nullptr;
        for (int q = 0; q < kMaxRanks; ++q) x.rows[q] = nullptr;
        if (!counts[k]) continue;
        uint32_t rb, re;
        shard(counts[k], &rb, &re);
        x.count = re - rb;
        if (mc) x.mc = mcs[k] + rb;
        for (int q = 0; q < world && !mc; ++q) {
            x.rows[q] = srcs[k][q] + rb;
            x.vec = x.vec && aligned16(x.rows[q]);
        }
        blocks += (x.count + kTileFloats - 1) / kTileFloats;
    }
    d.total_tiles = blocks;
    // Persistent grid: at most one wave of resident blocks; every rank launches
    // at least one block so that it signals and waits.
    auto kern = mc ? (world <= 2 ? dp_adam_kernel<2, true> : world <= 4 ? dp_adam_kernel<4, true>
                                                                       : dp_adam_kernel<8, true>)
                   : (world <= 2 ? dp_adam_kernel<2, false> : world <= 4 ? dp_adam_kernel<4, false>
                                                                         : dp_adam_kernel<8, false>);
    int sms = 0, per_sm = 0;
    bsx_status s = check_cuda(ctx, cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device),
                              "cudaDeviceGetAttribute");
    if (s == BSX_OK)
        s = check_cuda(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAdamThreads, 0),
                       "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (s != BSX_OK) return s;
    const uint32_t wave = (uint32_t)std::max(1, sms * std::max(1, per_sm));
    const uint32_t grid = std::max(1u, std::min(blocks, wave));
    prof_begin(ctx);
    kern<<<grid, kAdamThreads, 0, ctx->stream>>>(a);
    return post_launch(ctx, "dp_adam_kernel");
}
