// refine.cu - densification (prune / replace / split / grow) for the native trainer.
//
// Restates SplatTrainer::refine_for_phase, refine_splats and prune_points
// (crates/brush-train/src/train.rs:1191-1860) with the gradient-norm growth
// signal. Decisions and parameter arithmetic run on the device; only counts
// come back to the host. The split set is merged in the reference's order
// (replacement, oversized, growth) as flags over the kept rows.
//
//   plan:  refine_mask_kernel (prune predicates, train.rs:1258-1350) ->
//          ordered compaction of the kept ids (scan + scatter) ->
//          sample_keys_kernel + radix sort: weighted sampling without
//          replacement as the k largest Efraimidis-Spirakis keys log(u)/w
//          (u from SplitMix64 of seed, refine count, stream, index) ->
//          oversized candidates -> the split set as device flags (the
//          host sees only counts) -> ordered compaction of the split rows.
//   apply: gather_rows_kernel (kept rows of splats and Adam moments) ->
//          split_kernel (long-axis split of every selected splat, child
//          appended, both halves' moments zeroed, train.rs:1547-1700) ->
//          decay_kernel (opacity and scale decay, train.rs:1700-1740).
// Every per-element expression is evaluated in the reference's order, so the
// host restatement in the oracle matches bit for bit.
#include <algorithm>

#include "trainer.cuh"

namespace bsx {

namespace {

constexpr int kRefThreads = 256;

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform in (0, 1] with 24 random bits.
__device__ __forceinline__ float uniform01(uint64_t seed, uint32_t stream, uint32_t index) {
    const uint64_t h = splitmix64(seed ^ splitmix64(((uint64_t)stream << 32) | index));
    return (float)((h >> 40) + 1) * 5.9604644775390625e-08f;  // 2^-24
}

__device__ __forceinline__ float inv_sigmoid(float x) { return bsx_logf(x / (1.0f - x)); }  // train.rs:137-139
__device__ __forceinline__ float clampf(float x, float lo, float hi) { return bsx_min(bsx_max(x, lo), hi); }

struct MaskArgs {
    const float* t;
    const float* sh;
    const float* op;
    uint32_t n, c3;
    float min_opacity, max_allowed, min_scale_thr;
    float center[3];
    int radial, min_scale_prune, near_zero_rot;
    uint32_t* keep;      // [n] 1 = kept
    uint32_t* counters;  // [0] non-finite
};

__global__ void __launch_bounds__(kRefThreads) refine_mask_kernel(const __grid_constant__ MaskArgs a) {
    const uint32_t i = blockIdx.x * kRefThreads + threadIdx.x;
    bool bad = false;
    if (i < a.n) {
        const float* r = a.t + (size_t)i * 10;
        bool prune = bsx_sigmoid(a.op[i]) < a.min_opacity;
        bool big = false;
        for (int k = 0; k < 3; ++k) big |= bsx_expf(r[7 + k]) > a.max_allowed;
        prune |= big;
        bool out_b = false;
        if (a.radial) {
            const float dx = r[0] - a.center[0], dy = r[1] - a.center[1], dz = r[2] - a.center[2];
            out_b = sqrtf(dx * dx + dy * dy + dz * dz) > a.max_allowed;
        } else {
            for (int k = 0; k < 3; ++k) out_b |= fabsf(r[k] - a.center[k]) > a.max_allowed;
        }
        prune |= out_b;
        bad = !bsx_is_finite(a.op[i]);
        for (int k = 0; k < 10; ++k) bad |= !bsx_is_finite(r[k]);
        for (uint32_t k = 0; k < a.c3; ++k) bad |= !bsx_is_finite(a.sh[(size_t)i * a.c3 + k]);
        prune |= bad;
        if (a.min_scale_prune) {
            bool small = false;
            for (int k = 0; k < 3; ++k) small |= bsx_expf(r[7 + k]) < a.min_scale_thr;
            prune |= small;
        }
        if (a.near_zero_rot) prune |= (r[3] * r[3] + r[4] * r[4] + r[5] * r[5] + r[6] * r[6]) < 1e-8f;
        a.keep[i] = prune ? 0u : 1u;
    }
    const uint32_t nb = __popc(__ballot_sync(0xffffffffu, bad));
    if ((threadIdx.x & 31) == 0 && nb) atomicAdd(a.counters, nb);
}

// out[pos[i] - 1] = i for flagged i (pos: inclusive scan of the flags).
__global__ void __launch_bounds__(kRefThreads) scatter_flagged_kernel(const uint32_t* __restrict__ flag,
                                                                      const uint32_t* __restrict__ pos, uint32_t n,
                                                                      uint32_t* __restrict__ out) {
    const uint32_t i = blockIdx.x * kRefThreads + threadIdx.x;
    if (i < n && flag[i]) out[pos[i] - 1] = i;
}

__global__ void __launch_bounds__(kRefThreads) iota_kernel(uint32_t* out, uint32_t n) {
    const uint32_t i = blockIdx.x * kRefThreads + threadIdx.x;
    if (i < n) out[i] = i;
}

struct KeyArgs {
    const uint32_t* keep;  // kept original ids [K]
    uint32_t K;
    const float* op;       // splat logits (original numbering)
    const float* rn;       // RefineRecord (original numbering)
    const float* vis;
    int growth;            // 0: opacity x visibility, 1: gradient norm above the threshold
    float threshold;
    uint64_t seed;
    uint32_t stream;
    uint32_t* keys;        // |log(u)/w| bits, or all ones for w <= 0
    uint32_t* vals;        // kept index j
    uint32_t* counters;    // [0] positive weights, [1] above the threshold
};

__global__ void __launch_bounds__(kRefThreads) sample_keys_kernel(const __grid_constant__ KeyArgs a) {
    const uint32_t j = blockIdx.x * kRefThreads + threadIdx.x;
    bool pos = false, above = false;
    if (j < a.K) {
        const uint32_t i = a.keep[j];
        const float vis = a.vis[i];
        float w;
        if (a.growth) {
            above = a.rn[i] > a.threshold && vis > 0.0f;
            w = (above ? 1.0f : 0.0f) * a.rn[i];
        } else {
            w = bsx_sigmoid(a.op[i]) * (vis > 0.0f ? 1.0f : 0.0f);
        }
        pos = w > 0.0f && bsx_is_finite(w);
        uint32_t key = 0xffffffffu;
        if (pos) key = __float_as_uint(fabsf(bsx_logf(uniform01(a.seed, a.stream, j)) / w));
        a.keys[j] = key;
        a.vals[j] = j;
    }
    const uint32_t np = __popc(__ballot_sync(0xffffffffu, pos));
    const uint32_t na = __popc(__ballot_sync(0xffffffffu, above));
    if ((threadIdx.x & 31) == 0) {
        if (np) atomicAdd(a.counters, np);
        if (na) atomicAdd(a.counters + 1, na);
    }
}

// Marks the first `take` sampled rows as split (no duplicates within one draw);
// counts the rows that were not marked before.
__global__ void __launch_bounds__(kRefThreads) mark_sampled_kernel(const uint32_t* __restrict__ vals, uint32_t take,
                                                                   uint32_t* __restrict__ mark,
                                                                   uint32_t* __restrict__ fresh) {
    const uint32_t i = blockIdx.x * kRefThreads + threadIdx.x;
    bool is_new = false;
    if (i < take) {
        const uint32_t j = vals[i];
        is_new = mark[j] == 0u;
        mark[j] = 1u;
    }
    const uint32_t c = __popc(__ballot_sync(0xffffffffu, is_new));
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(fresh, c);
}

// Oversized candidates not yet in the split set, in row order.
__global__ void __launch_bounds__(kRefThreads) oversized_new_kernel(const uint32_t* __restrict__ keep, uint32_t K,
                                                                    const float* __restrict__ screen,
                                                                    const float* __restrict__ vis, float thr,
                                                                    const uint32_t* __restrict__ mark,
                                                                    uint32_t* __restrict__ flag) {
    const uint32_t j = blockIdx.x * kRefThreads + threadIdx.x;
    if (j < K) {
        const uint32_t i = keep[j];
        flag[j] = (screen[i] > thr && vis[i] > 0.0f && mark[j] == 0u) ? 1u : 0u;
    }
}

// The first `budget` new candidates join the split set (train.rs:1410-1421).
__global__ void __launch_bounds__(kRefThreads) mark_budget_kernel(const uint32_t* __restrict__ flag,
                                                                  const uint32_t* __restrict__ pos, uint32_t K,
                                                                  uint32_t budget, uint32_t* __restrict__ mark) {
    const uint32_t j = blockIdx.x * kRefThreads + threadIdx.x;
    if (j < K && flag[j] && pos[j] <= budget) mark[j] = 1u;
}

// dst[j, :] = src[idx[j], :] for j < rows (cols floats per row).
__global__ void __launch_bounds__(kRefThreads) gather_rows_kernel(const float* __restrict__ src,
                                                                  const uint32_t* __restrict__ idx, uint32_t rows,
                                                                  uint32_t cols, float* __restrict__ dst) {
    const uint64_t e = (uint64_t)blockIdx.x * kRefThreads + threadIdx.x;
    if (e >= (uint64_t)rows * cols) return;
    const uint32_t j = (uint32_t)(e / cols), c = (uint32_t)(e - (uint64_t)j * cols);
    dst[e] = src[(size_t)idx[j] * cols + c];
}

struct SplitArgs {
    const uint32_t* split;  // kept-numbering rows, ascending [S]
    const uint32_t* keep;   // kept original ids (for the screen size)
    const float* screen;    // RefineRecord max_screen_size (original numbering)
    uint32_t S, K, c3;
    float* t;               // new splats [K+S] (rows < K already gathered)
    float* sh;
    float* op;
    float* m[3];            // new moments
    float* v[3];
    float split_at, long_scale, other_scale, opac_scale, min_opacity;
};

// train.rs:1547-1700 for one selected splat.
__global__ void __launch_bounds__(kRefThreads) split_kernel(const __grid_constant__ SplitArgs a) {
    const uint32_t q = blockIdx.x * kRefThreads + threadIdx.x;
    if (q >= a.S) return;
    const uint32_t s = a.split[q], child = a.K + q;
    float* pr = a.t + (size_t)s * 10;
    const float mean[3] = {pr[0], pr[1], pr[2]};
    const float qr[4] = {pr[3], pr[4], pr[5], pr[6]};
    const float ls[3] = {pr[7], pr[8], pr[9]};
    const float raw_op = a.op[s];
    const float mag = bsx_max(sqrtf(qr[0] * qr[0] + qr[1] * qr[1] + qr[2] * qr[2] + qr[3] * qr[3]), 1e-32f);
    const float rot[4] = {qr[0] / mag, qr[1] / mag, qr[2] / mag, qr[3] / mag};
    const float sc[3] = {bsx_expf(ls[0]), bsx_expf(ls[1]), bsx_expf(ls[2])};
    const float new_opac = bsx_sigmoid(raw_op) * a.opac_scale;
    const float new_raw = inv_sigmoid(clampf(new_opac, a.min_opacity, 1.0f - a.min_opacity));
    int L = 0;
    for (int k = 1; k < 3; ++k)
        if (ls[k] > ls[L]) L = k;
    float m_long = a.long_scale;
    if (a.split_at > 0.0f)
        m_long = bsx_min((1.0f / bsx_max(a.screen[a.keep[s]], 1e-6f)) * a.split_at, a.long_scale);
    float off[3];
    for (int k = 0; k < 3; ++k) off[k] = ((k == L ? 1.0f : 0.0f) * sc[k]) * a.long_scale;
    const float qw = rot[0], qx = rot[1], qy = rot[2], qz = rot[3];
    const float vx = off[0], vy = off[1], vz = off[2];
    const float qw2 = qw * qw, qx2 = qx * qx, qy2 = qy * qy, qz2 = qz * qz;
    const float xy = qx * qy, xz = qx * qz, yz = qy * qz, wx = qw * qx, wy = qw * qy, wz = qw * qz;
    const float smp[3] = {
        (qw2 + qx2 - qy2 - qz2) * vx + (xy * vy + xz * vz + wy * vz - wz * vy) * 2.0f,
        (qw2 - qx2 + qy2 - qz2) * vy + (xy * vx + yz * vz + wz * vx - wx * vz) * 2.0f,
        (qw2 - qx2 - qy2 + qz2) * vz + (xz * vx + yz * vy + wx * vy - wy * vx) * 2.0f};
    const float ln_other = bsx_logf(a.other_scale), ln_long = bsx_logf(m_long);
    float nls[3];
    for (int k = 0; k < 3; ++k) {
        const float oh = k == L ? 1.0f : 0.0f;
        const float base = ls[k] + ln_other, lng = ls[k] + ln_long;
        nls[k] = base * (-oh + 1.0f) + lng * oh;
    }
    for (int k = 0; k < 3; ++k) {
        pr[k] = mean[k] + (-smp[k]);
        pr[7 + k] = ls[k] + (nls[k] - ls[k]);
    }
    for (int k = 0; k < 4; ++k) pr[3 + k] = qr[k] + 0.0f;
    a.op[s] = raw_op + (new_raw - raw_op);
    float* cr = a.t + (size_t)child * 10;
    for (int k = 0; k < 3; ++k) cr[k] = mean[k] + smp[k];
    for (int k = 0; k < 4; ++k) cr[3 + k] = rot[k];
    for (int k = 0; k < 3; ++k) cr[7 + k] = nls[k];
    for (uint32_t k = 0; k < a.c3; ++k) a.sh[(size_t)child * a.c3 + k] = a.sh[(size_t)s * a.c3 + k];
    a.op[child] = new_raw;
    // both halves start with zero moments (the parent as x + (-x), train.rs:1684-1725)
    const uint32_t cols[3] = {10, a.c3, 1};
    for (int g = 0; g < 3; ++g) {
        float* m = a.m[g];
        for (uint32_t k = 0; k < cols[g]; ++k) {
            m[(size_t)s * cols[g] + k] = m[(size_t)s * cols[g] + k] + (-m[(size_t)s * cols[g] + k]);
            m[(size_t)child * cols[g] + k] = 0.0f;
        }
    }
    const uint32_t vcols[3] = {10, 1, 1};
    for (int g = 0; g < 3; ++g) {
        float* v = a.v[g];
        for (uint32_t k = 0; k < vcols[g]; ++k) {
            v[(size_t)s * vcols[g] + k] = v[(size_t)s * vcols[g] + k] + (-v[(size_t)s * vcols[g] + k]);
            v[(size_t)child * vcols[g] + k] = 0.0f;
        }
    }
}

// train.rs:1700-1740: opacity decay, and scale decay when enabled.
__global__ void __launch_bounds__(kRefThreads) decay_kernel(float* __restrict__ t, float* __restrict__ op,
                                                            uint32_t rows, float minus_opac, float scale_factor,
                                                            int scale_decay) {
    const uint32_t r = blockIdx.x * kRefThreads + threadIdx.x;
    if (r >= rows) return;
    const float new_op = bsx_sigmoid(op[r]) - minus_opac;
    op[r] = inv_sigmoid(clampf(new_op, 1e-12f, 1.0f - 1e-12f));
    if (scale_decay)
        for (int k = 0; k < 3; ++k) {
            float* v = t + (size_t)r * 10 + 7 + k;
            *v = bsx_logf(bsx_max(bsx_expf(*v) * scale_factor, 1e-12f));
        }
}

// ---- gradient-threshold rule (the original 3DGS densify_and_clone / densify_and_split) ----

// Selection of the kept rows: average view-space gradient norm over the
// visible steps >= threshold; clone where the largest scale is at most `dense`,
// split otherwise.
__global__ void __launch_bounds__(kRefThreads)
    grad_select_kernel(const uint32_t* __restrict__ keep, uint32_t K, const float* __restrict__ t,
                       const float* __restrict__ vis, const float* __restrict__ grad2d, float threshold, float dense,
                       uint32_t* __restrict__ clone_flag, uint32_t* __restrict__ split_flag) {
    const uint32_t j = blockIdx.x * kRefThreads + threadIdx.x;
    if (j >= K) return;
    const uint32_t i = keep[j];
    const float avg = vis[i] > 0.0f ? grad2d[i] / vis[i] : 0.0f;
    const bool sel = avg >= threshold;
    const float* r = t + (size_t)i * 10;
    const float smax = bsx_max(bsx_max(bsx_expf(r[7]), bsx_expf(r[8])), bsx_expf(r[9]));
    clone_flag[j] = (sel && smax <= dense) ? 1u : 0u;
    split_flag[j] = (sel && !(smax <= dense)) ? 1u : 0u;
}

// out[pos[j] - 1] = j for the first `limit` flagged rows; taken[j] marks them.
__global__ void __launch_bounds__(kRefThreads)
    take_first_kernel(const uint32_t* __restrict__ flag, const uint32_t* __restrict__ pos, uint32_t K, uint32_t limit,
                      uint32_t* __restrict__ out, uint32_t* __restrict__ taken) {
    const uint32_t j = blockIdx.x * kRefThreads + threadIdx.x;
    if (j >= K) return;
    const bool t = flag[j] && pos[j] <= limit;
    if (t) out[pos[j] - 1] = j;
    if (taken) taken[j] = t ? 0u : 1u;  // 1 = stays (not split)
}

// idx2[r] = keep[idx[r]] (kept numbering -> original ids).
__global__ void __launch_bounds__(kRefThreads) compose_kernel(const uint32_t* __restrict__ keep,
                                                              const uint32_t* __restrict__ idx, uint32_t count,
                                                              uint32_t* __restrict__ out) {
    const uint32_t r = blockIdx.x * kRefThreads + threadIdx.x;
    if (r < count) out[r] = keep[idx[r]];
}

struct GtSplitArgs {
    const uint32_t* split;  // split rows (kept numbering) [S]
    const uint32_t* keep;   // kept original ids
    const float* t;         // old splats
    const float* sh;
    const float* op;
    float* nt;              // rows `base`.. receive the children
    float* nsh;
    float* nop;
    uint32_t S, c3, base, refine_count;
    uint64_t seed;
};

// Child k of split row q at row base + k S + q: mean + R(q) (s * n), log(s / 1.6),
// rotation, SH and opacity copied (the original 3DGS densify_and_split, N = 2).
__global__ void __launch_bounds__(kRefThreads) grad_split_kernel(const __grid_constant__ GtSplitArgs a) {
    const uint32_t e = blockIdx.x * kRefThreads + threadIdx.x;
    if (e >= 2 * a.S) return;
    const uint32_t k = e / a.S, q = e - k * a.S;
    const uint32_t j = a.split[q], i = a.keep[j], r = a.base + e;
    const float* pr = a.t + (size_t)i * 10;
    const float mag = bsx_max(sqrtf(pr[3] * pr[3] + pr[4] * pr[4] + pr[5] * pr[5] + pr[6] * pr[6]), 1e-32f);
    const float qw = pr[3] / mag, qx = pr[4] / mag, qy = pr[5] / mag, qz = pr[6] / mag;
    float z[3];
    bsx_normal3(a.seed, (1u << 30) + 2 * a.refine_count + k, j, z);
    const float vx = bsx_expf(pr[7]) * z[0], vy = bsx_expf(pr[8]) * z[1], vz = bsx_expf(pr[9]) * z[2];
    const float qw2 = qw * qw, qx2 = qx * qx, qy2 = qy * qy, qz2 = qz * qz;
    const float xy = qx * qy, xz = qx * qz, yz = qy * qz, wx = qw * qx, wy = qw * qy, wz = qw * qz;
    const float d[3] = {(qw2 + qx2 - qy2 - qz2) * vx + (xy * vy + xz * vz + wy * vz - wz * vy) * 2.0f,
                        (qw2 - qx2 + qy2 - qz2) * vy + (xy * vx + yz * vz + wz * vx - wx * vz) * 2.0f,
                        (qw2 - qx2 - qy2 + qz2) * vz + (xz * vx + yz * vy + wx * vy - wy * vx) * 2.0f};
    float* cr = a.nt + (size_t)r * 10;
    for (int c = 0; c < 3; ++c) cr[c] = pr[c] + d[c];
    for (int c = 0; c < 4; ++c) cr[3 + c] = pr[3 + c];
    for (int c = 0; c < 3; ++c) cr[7 + c] = bsx_logf(bsx_expf(pr[7 + c]) / 1.6f);
    for (uint32_t c = 0; c < a.c3; ++c) a.nsh[(size_t)r * a.c3 + c] = a.sh[(size_t)i * a.c3 + c];
    a.nop[r] = a.op[i];
}

uint32_t blocks_for(uint64_t n) { return (uint32_t)((n + kRefThreads - 1) / kRefThreads); }

// Reads `count` u32 from the device (synchronises the stream).
bsx_status read_u32(bsx_ctx* ctx, const uint32_t* d, uint32_t count, uint32_t* h) {
    if (count == 0) return BSX_OK;
    bsx_status s = check_cuda(ctx, cudaMemcpyAsync(h, d, (size_t)count * 4, cudaMemcpyDeviceToHost, ctx->stream),
                              "refine readback");
    if (s != BSX_OK) return s;
    return check_device_error(ctx);
}

// Weighted sample without replacement of up to k kept rows (stream picks the
// draw); the drawn rows are marked in `mark`. Returns through `drawn_new` how
// many of them were not marked before, and through `above_count` the rows
// above the growth threshold.
bsx_status weighted_sample(bsx_trainer* tr, const float* op, int growth, uint32_t k, uint32_t stream,
                           uint32_t* scratch, uint32_t* mark, uint32_t* above_count, uint32_t* drawn_new) {
    bsx_ctx* ctx = tr->ctx;
    const uint32_t K = tr->plan_kept, n = tr->plan_n;
    float* st = tr->stats.as<float>();
    uint32_t* keys = scratch;
    uint32_t* vals = keys + n;
    uint32_t* keys_out = vals + n;
    uint32_t* vals_out = keys_out + n;
    uint32_t* counters = scratch + (size_t)n * 5 + 8;
    bsx_status s = check_cuda(ctx, cudaMemsetAsync(counters, 0, 12, ctx->stream), "memset sample counters");
    if (s != BSX_OK) return s;
    KeyArgs a;
    a.keep = tr->plan_keep.as<uint32_t>();
    a.K = K;
    a.op = op;
    a.rn = st;
    a.vis = st + tr->n;
    a.growth = growth;
    a.threshold = tr->plan_cfg.growth_grad_threshold;
    a.seed = tr->plan_cfg.seed;
    a.stream = stream;
    a.keys = keys;
    a.vals = vals;
    a.counters = counters;
    if (K) {
        prof_begin(ctx);
        sample_keys_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(a);
        s = post_launch(ctx, "sample_keys_kernel");
        if (s != BSX_OK) return s;
    }
    uint32_t c[2] = {0, 0};
    s = read_u32(ctx, counters, 2, c);
    if (s != BSX_OK) return s;
    if (above_count) *above_count = c[1];
    if (drawn_new) *drawn_new = 0;
    const uint32_t take = std::min(k, c[0]);
    if (take == 0) return BSX_OK;
    s = radix_sort_pairs(ctx, keys, vals, K, 32, keys_out, vals_out);
    if (s != BSX_OK) return s;
    prof_begin(ctx);
    mark_sampled_kernel<<<blocks_for(take), kRefThreads, 0, ctx->stream>>>(vals_out, take, mark, counters + 2);
    s = post_launch(ctx, "mark_sampled_kernel");
    if (s == BSX_OK && drawn_new) s = read_u32(ctx, counters + 2, 1, drawn_new);
    return s;
}

uint32_t sat_sub(uint32_t a, uint32_t b) { return a > b ? a - b : 0u; }

}  // namespace

}  // namespace bsx

using namespace bsx;

extern "C" bsx_status bsx_trainer_refine_plan(bsx_trainer* tr, const float* t, const float* sh, const float* op,
                                              const bsx_refine_config* cfg, const float center[3],
                                              const float extent[3], uint32_t global_iter, bsx_refine_stats* stats) {
    if (!tr || !cfg || !center || !extent || (tr->n && (!t || !sh || !op))) return BSX_ERR_INVALID_ARG;
    bsx_ctx* ctx = tr->ctx;
    if (tr->moment_world > 1)
        return fail(ctx, BSX_ERR_UNSUPPORTED, "refine with sharded data-parallel optimizer state is not built");
    if (!tr->cfg.gather_stats) return fail(ctx, BSX_ERR_STATE, "refine needs a trainer created with gather_stats");
    cudaSetDevice(ctx->device);
    tr->planned = false;
    const uint32_t n = tr->n, c3 = 3 * tr->coeffs;
    tr->plan_n = n;
    tr->plan_cfg = *cfg;
    bsx_status s = ensure(ctx, tr->plan_keep, ((size_t)n + 1) * 4);
    // scratch (u32): four arrays of n (mask / positions / sort keys and values), counters at 5n,
    // then the split membership of the kept rows at 5n + 32
    if (s == BSX_OK) s = ensure(ctx, tr->plan_scratch, ((size_t)n * 6 + 32) * 4);
    if (s != BSX_OK) return s;
    uint32_t* scratch = tr->plan_scratch.as<uint32_t>();
    uint32_t* flag = scratch;
    uint32_t* pos = flag + n;
    uint32_t* counters = scratch + (size_t)n * 5;
    uint32_t* keep = tr->plan_keep.as<uint32_t>();
    s = check_cuda(ctx, cudaMemsetAsync(counters, 0, 32 * 4, ctx->stream), "memset refine counters");
    if (s != BSX_OK) return s;
    const float max_extent = bsx_max(bsx_max(extent[0], extent[1]), extent[2]);
    uint32_t K = 0, non_finite = 0;
    if (n) {
        MaskArgs a;
        a.t = t;
        a.sh = sh;
        a.op = op;
        a.n = n;
        a.c3 = c3;
        a.min_opacity = cfg->min_opacity;
        a.max_allowed = max_extent * cfg->prune_extent_factor;
        a.min_scale_thr = cfg->min_scale_prune_threshold;
        for (int k = 0; k < 3; ++k) a.center[k] = center[k];
        a.radial = cfg->radial_bounds_prune;
        a.min_scale_prune = cfg->min_scale_prune;
        a.near_zero_rot = cfg->near_zero_rotation_prune;
        a.keep = flag;
        a.counters = counters;
        prof_begin(ctx);
        refine_mask_kernel<<<blocks_for(n), kRefThreads, 0, ctx->stream>>>(a);
        s = post_launch(ctx, "refine_mask_kernel");
        if (s == BSX_OK) s = scan_inclusive_u32(ctx, flag, nullptr, n, pos, counters + 1);
        if (s != BSX_OK) return s;
        prof_begin(ctx);
        scatter_flagged_kernel<<<blocks_for(n), kRefThreads, 0, ctx->stream>>>(flag, pos, n, keep);
        s = post_launch(ctx, "scatter_flagged_kernel");
        if (s != BSX_OK) return s;
        uint32_t c[2];
        s = read_u32(ctx, counters, 2, c);
        if (s != BSX_OK) return s;
        non_finite = c[0];
        K = c[1];
        if (K == 0) {  // prune_points keeps every splat when all would go (train.rs:1830-1833)
            prof_begin(ctx);
            iota_kernel<<<blocks_for(n), kRefThreads, 0, ctx->stream>>>(keep, n);
            s = post_launch(ctx, "iota_kernel");
            if (s != BSX_OK) return s;
            K = n;
        }
    }
    tr->plan_kept = K;
    const uint32_t pruned = n - K;
    if (cfg->rule == BSX_REFINE_GRAD_THRESHOLD) {
        if (!tr->cfg.accumulate_grad2d)
            return fail(ctx, BSX_ERR_STATE, "the gradient-threshold rule needs a trainer with accumulate_grad2d");
        // scratch (u32): [0, n) flags, [n, 2n) positions, [2n, 3n) clone rows, [3n, 4n) rows that stay,
        // [4n, 5n) their positions, counters at 5n, the stay flags at 5n + 32
        float* st = tr->stats.as<float>();
        uint32_t* cflag = scratch;
        uint32_t* cpos = scratch + n;
        uint32_t* clone_rows = scratch + 2 * (size_t)n;
        uint32_t* stay_rows = scratch + 3 * (size_t)n;
        uint32_t* stay_pos = scratch + 4 * (size_t)n;
        uint32_t* stay = scratch + (size_t)n * 5 + 32;
        uint32_t* sflag = stay;  // split flags first, then (take_first) the stay flags
        s = ensure(ctx, tr->plan_split, ((size_t)K + 1) * 4);
        if (s != BSX_OK) return s;
        uint32_t* split_rows = tr->plan_split.as<uint32_t>();
        uint32_t cand[2] = {0, 0};
        if (K) {
            const float dense = cfg->percent_dense * max_extent;
            prof_begin(ctx);
            grad_select_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(
                keep, K, t, st + tr->n, st + 3 * (size_t)tr->n, cfg->growth_grad_threshold, dense, cflag, sflag);
            s = post_launch(ctx, "grad_select_kernel");
            if (s == BSX_OK) s = scan_inclusive_u32(ctx, cflag, nullptr, K, cpos, counters + 2);
            if (s == BSX_OK) s = scan_inclusive_u32(ctx, sflag, nullptr, K, stay_pos, counters + 3);
            if (s == BSX_OK) s = read_u32(ctx, counters + 2, 2, cand);
            if (s != BSX_OK) return s;
        }
        uint32_t budget = sat_sub(cfg->max_splats, K);
        const uint32_t C = std::min(cand[0], budget);
        budget -= C;
        const uint32_t S = std::min(cand[1], budget);
        if (K) {
            prof_begin(ctx);
            take_first_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(cflag, cpos, K, C, clone_rows, nullptr);
            s = post_launch(ctx, "take_first_kernel");
            if (s != BSX_OK) return s;
            prof_begin(ctx);
            // split rows in order; the flags become "stays" (1 = not split)
            take_first_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(sflag, stay_pos, K, S, split_rows, stay);
            s = post_launch(ctx, "take_first_kernel");
            if (s == BSX_OK) s = scan_inclusive_u32(ctx, stay, nullptr, K, stay_pos, nullptr);
            if (s != BSX_OK) return s;
            prof_begin(ctx);
            scatter_flagged_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(stay, stay_pos, K, stay_rows);
            s = post_launch(ctx, "scatter_flagged_kernel");
            if (s != BSX_OK) return s;
        }
        tr->plan_clone_count = C;
        tr->plan_split_count = S;
        tr->planned = true;
        if (stats) {
            stats->num_added = C + S;
            stats->num_split_oversized = 0;
            stats->num_split_high_grad = S;
            stats->num_pruned = pruned;
            stats->num_pruned_non_finite = non_finite;
            stats->total_splats = K + C + S;
        }
        return BSX_OK;
    }
    const uint32_t stream0 = 2 * tr->refines;
    // split membership of the kept rows; the reference's HashSet (train.rs:1366)
    uint32_t* mark = scratch + (size_t)n * 5 + 32;
    uint32_t* sample_scratch = scratch;  // the mask and positions are no longer needed
    if (K) {
        s = check_cuda(ctx, cudaMemsetAsync(mark, 0, (size_t)K * 4, ctx->stream), "memset split set");
        if (s != BSX_OK) return s;
    }
    uint32_t in_set = 0;
    if (pruned > 0) {  // replacement weighted by opacity x visibility (train.rs:1368-1392)
        uint32_t fresh = 0;
        s = weighted_sample(tr, op, 0, pruned, stream0, sample_scratch, mark, nullptr, &fresh);
        if (s != BSX_OK) return s;
        in_set += fresh;
    }
    uint32_t num_oversized = 0;
    if (cfg->split_at_screen_size > 0.0f && K) {  // train.rs:1398-1424
        float* st = tr->stats.as<float>();
        uint32_t* oflag = scratch;
        uint32_t* opos = oflag + n;
        uint32_t* ocount = scratch + (size_t)n * 5 + 4;
        prof_begin(ctx);
        oversized_new_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(
            keep, K, st + 2 * (size_t)tr->n, st + tr->n, cfg->split_at_screen_size, mark, oflag);
        s = post_launch(ctx, "oversized_new_kernel");
        if (s == BSX_OK) s = scan_inclusive_u32(ctx, oflag, nullptr, K, opos, ocount);
        uint32_t fresh_candidates = 0;
        if (s == BSX_OK) s = read_u32(ctx, ocount, 1, &fresh_candidates);
        if (s != BSX_OK) return s;
        const uint32_t budget = sat_sub(cfg->max_splats, K + in_set);
        num_oversized = std::min(budget, fresh_candidates);
        if (num_oversized) {
            prof_begin(ctx);
            mark_budget_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(oflag, opos, K, budget, mark);
            s = post_launch(ctx, "mark_budget_kernel");
            if (s != BSX_OK) return s;
        }
        in_set += num_oversized;
    }
    uint32_t num_high_grad = 0;
    if (global_iter < cfg->growth_stop_iter && K) {  // train.rs:1428-1495, gradient signal
        // count the candidates first (k = 0 draws nothing), then draw
        uint32_t count = 0;
        s = weighted_sample(tr, op, 1, 0, stream0 + 1, sample_scratch, mark, &count, nullptr);
        if (s != BSX_OK) return s;
        const uint32_t grow_count = (uint32_t)roundf((float)count * cfg->growth_select_fraction);
        const uint32_t sample_high = sat_sub(grow_count, pruned);
        const uint32_t headroom = sat_sub(cfg->max_splats, K + in_set);
        const uint32_t grow = std::min(sample_high, headroom);
        if (grow > 0) {
            s = weighted_sample(tr, op, 1, grow, stream0 + 1, sample_scratch, mark, nullptr, &num_high_grad);
            if (s != BSX_OK) return s;
            in_set += num_high_grad;
        }
    }
    // the split rows in ascending order
    const uint32_t S = in_set;
    s = ensure(ctx, tr->plan_split, ((size_t)K + 1) * 4);
    if (s != BSX_OK) return s;
    if (S) {
        uint32_t* mpos = scratch;
        s = scan_inclusive_u32(ctx, mark, nullptr, K, mpos, nullptr);
        if (s != BSX_OK) return s;
        prof_begin(ctx);
        scatter_flagged_kernel<<<blocks_for(K), kRefThreads, 0, ctx->stream>>>(mark, mpos, K,
                                                                               tr->plan_split.as<uint32_t>());
        s = post_launch(ctx, "scatter_flagged_kernel");
        if (s != BSX_OK) return s;
    }
    tr->plan_split_count = S;
    tr->planned = true;
    if (stats) {
        stats->num_added = S;
        stats->num_split_oversized = num_oversized;
        stats->num_split_high_grad = num_high_grad;
        stats->num_pruned = pruned;
        stats->num_pruned_non_finite = non_finite;
        stats->total_splats = K + S;
    }
    return BSX_OK;
}

extern "C" bsx_status bsx_trainer_refine_apply(bsx_trainer* tr, const float* t, const float* sh, const float* op,
                                               float* nt, float* nsh, float* nop, uint32_t phase_iter,
                                               uint32_t phase_total) {
    if (!tr) return BSX_ERR_INVALID_ARG;
    bsx_ctx* ctx = tr->ctx;
    if (!tr->planned) return fail(ctx, BSX_ERR_STATE, "bsx_trainer_refine_apply needs a fresh bsx_trainer_refine_plan");
    const bsx_refine_config& cfg = tr->plan_cfg;
    const bool gt_rule = cfg.rule == BSX_REFINE_GRAD_THRESHOLD;
    const uint32_t C = gt_rule ? tr->plan_clone_count : 0;
    const uint32_t K = tr->plan_kept, S = tr->plan_split_count, N2 = K + S + C, n = tr->n, c3 = 3 * tr->coeffs;
    if (N2 && (!t || !sh || !op || !nt || !nsh || !nop)) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    // old moments (zeros if no optimizer step has been taken yet)
    float* m_old[3];
    float* v_old[3];
    bsx_status s = ensure(ctx, tr->moments, moment_floats(n, tr->coeffs) * 4 + 64);
    if (s != BSX_OK) return s;
    if (tr->moment_rows != n || tr->moment_world != 1) {
        s = check_cuda(ctx, cudaMemsetAsync(tr->moments.p, 0, moment_floats(n, tr->coeffs) * 4, ctx->stream),
                       "memset moments");
        if (s != BSX_OK) return s;
    }
    moment_views(tr->moments.as<float>(), n, tr->coeffs, m_old, v_old);
    s = ensure(ctx, tr->moments_next, moment_floats(N2, tr->coeffs) * 4 + 64);
    if (s != BSX_OK) return s;
    float* m_new[3];
    float* v_new[3];
    moment_views(tr->moments_next.as<float>(), N2, tr->coeffs, m_new, v_new);
    const uint32_t* keep = tr->plan_keep.as<uint32_t>();
    struct G {
        const float* src;
        float* dst;
        uint32_t cols;
    } gathers[9] = {{t, nt, 10},         {sh, nsh, c3},       {op, nop, 1},
                    {m_old[0], m_new[0], 10}, {m_old[1], m_new[1], c3}, {m_old[2], m_new[2], 1},
                    {v_old[0], v_new[0], 10}, {v_old[1], v_new[1], 1},  {v_old[2], v_new[2], 1}};
    if (gt_rule) {
        // rows: the K - S kept rows that stay, C clones, S first children, S second children;
        // new rows start with zero moments
        uint32_t* scratch = tr->plan_scratch.as<uint32_t>();
        uint32_t* stay_rows = scratch + 3 * (size_t)n;
        uint32_t* orig = scratch;  // original ids of the stays, then of the clones
        const uint32_t K2 = K - S;
        s = check_cuda(ctx, cudaMemsetAsync(tr->moments_next.p, 0, moment_floats(N2, tr->coeffs) * 4, ctx->stream),
                       "memset new moments");
        if (s != BSX_OK) return s;
        if (K2) {
            prof_begin(ctx);
            compose_kernel<<<blocks_for(K2), kRefThreads, 0, ctx->stream>>>(keep, stay_rows, K2, orig);
            s = post_launch(ctx, "compose_kernel");
            if (s != BSX_OK) return s;
            for (const G& g : gathers) {
                prof_begin(ctx);
                gather_rows_kernel<<<blocks_for((uint64_t)K2 * g.cols), kRefThreads, 0, ctx->stream>>>(g.src, orig, K2,
                                                                                                       g.cols, g.dst);
                s = post_launch(ctx, "gather_rows_kernel");
                if (s != BSX_OK) return s;
            }
        }
        if (C) {
            prof_begin(ctx);
            compose_kernel<<<blocks_for(C), kRefThreads, 0, ctx->stream>>>(keep, scratch + 2 * (size_t)n, C, orig);
            s = post_launch(ctx, "compose_kernel");
            if (s != BSX_OK) return s;
            for (int k = 0; k < 3; ++k) {
                const G& g = gathers[k];
                prof_begin(ctx);
                gather_rows_kernel<<<blocks_for((uint64_t)C * g.cols), kRefThreads, 0, ctx->stream>>>(
                    g.src, orig, C, g.cols, g.dst + (size_t)K2 * g.cols);
                s = post_launch(ctx, "gather_rows_kernel");
                if (s != BSX_OK) return s;
            }
        }
        if (S) {
            GtSplitArgs a;
            a.split = tr->plan_split.as<uint32_t>();
            a.keep = keep;
            a.t = t;
            a.sh = sh;
            a.op = op;
            a.nt = nt;
            a.nsh = nsh;
            a.nop = nop;
            a.S = S;
            a.c3 = c3;
            a.base = K2 + C;
            a.refine_count = tr->refines;
            a.seed = cfg.seed;
            prof_begin(ctx);
            grad_split_kernel<<<blocks_for(2 * (uint64_t)S), kRefThreads, 0, ctx->stream>>>(a);
            s = post_launch(ctx, "grad_split_kernel");
            if (s != BSX_OK) return s;
        }
    }
    if (K && !gt_rule)
        for (const G& g : gathers) {
            prof_begin(ctx);
            gather_rows_kernel<<<blocks_for((uint64_t)K * g.cols), kRefThreads, 0, ctx->stream>>>(g.src, keep, K,
                                                                                                  g.cols, g.dst);
            s = post_launch(ctx, "gather_rows_kernel");
            if (s != BSX_OK) return s;
        }
    if (S && !gt_rule) {
        SplitArgs a;
        a.split = tr->plan_split.as<uint32_t>();
        a.keep = keep;
        a.screen = tr->stats.as<float>() + 2 * (size_t)n;
        a.S = S;
        a.K = K;
        a.c3 = c3;
        a.t = nt;
        a.sh = nsh;
        a.op = nop;
        for (int g = 0; g < 3; ++g) {
            a.m[g] = m_new[g];
            a.v[g] = v_new[g];
        }
        a.split_at = cfg.split_at_screen_size;
        a.long_scale = cfg.split_long_axis_scale;
        a.other_scale = cfg.split_other_axis_scale;
        a.opac_scale = cfg.split_opacity_scale;
        a.min_opacity = cfg.min_opacity;
        prof_begin(ctx);
        split_kernel<<<blocks_for(S), kRefThreads, 0, ctx->stream>>>(a);
        s = post_launch(ctx, "split_kernel");
        if (s != BSX_OK) return s;
    }
    if (N2 && !gt_rule) {
        const float train_t = bsx_min(bsx_max((float)phase_iter / (float)std::max(phase_total, 1u), 0.0f), 1.0f);
        const float t_shrink = 1.0f - train_t;
        prof_begin(ctx);
        decay_kernel<<<blocks_for(N2), kRefThreads, 0, ctx->stream>>>(nt, nop, N2, cfg.opac_decay * t_shrink,
                                                                      1.0f - cfg.scale_decay * t_shrink,
                                                                      cfg.scale_decay > 0.0f);
        s = post_launch(ctx, "decay_kernel");
        if (s != BSX_OK) return s;
    }
    // the trainer now describes N2 splats: moments swapped in, a fresh RefineRecord
    std::swap(tr->moments, tr->moments_next);
    tr->moment_rows = N2;
    tr->moment_world = 1;
    tr->moment_rank = 0;
    tr->n = N2;
    const size_t nn = N2 ? N2 : 1;
    s = ensure(ctx, tr->v_combined, nn * BSX_GRAD_STRIDE * 4);
    if (s == BSX_OK) s = ensure(ctx, tr->stats, kRecordArrays * nn * 4);
    if (s == BSX_OK)
        s = check_cuda(ctx, cudaMemsetAsync(tr->stats.p, 0, kRecordArrays * nn * 4, ctx->stream),
                       "reset refine record");
    if (s != BSX_OK) return s;
    tr->planned = false;
    tr->refines++;
    return BSX_OK;
}
