// sort.cu - stable LSD radix argsort of u32 keys with u32 values.
//
// Replaces brush-sort (crates/brush-sort/src/lib.rs:16-129, kernels.rs:28-443:
// 4-bit digits, five kernels per pass). Here: one histogram kernel reads the
// keys once for every pass, then one kernel per 8-bit digit pass ("onesweep",
// Adinets & Merrill 2022): each 4096-key tile takes a ticket, ranks its keys
// stably with a warp-level ballot multi-split (the lanes holding the same
// digit are found by one ballot per digit bit, cheaper here than a match
// instruction), publishes its per-digit counts, looks back over
// predecessors' per-digit prefixes (bounded waits), and scatters through
// shared memory so that global writes are runs of consecutive addresses. The
// pass is register-bounded to four resident blocks per SM (64 registers):
// occupancy, not arithmetic, sets its speed.
//
// Semantics match the reference: the order is by (key & mask) where mask
// keeps ceil(bits/4)*4 low bits; equal keys keep their input order; the
// input arrays are not modified.
#include <algorithm>

#include "common.cuh"

namespace bsx {

namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;
constexpr uint32_t kSortTile = kSortThreads * kSortItems;  // 4096
constexpr int kRadix = 256;
constexpr uint32_t kLbAgg = 1u << 30;
constexpr uint32_t kLbIncl = 2u << 30;
constexpr uint32_t kLbMask = (1u << 30) - 1u;
constexpr int kMaxPasses = 4;

__global__ void __launch_bounds__(kSortThreads) sort_hist_kernel(const uint32_t* __restrict__ keys, uint32_t n,
                                                                 uint32_t mask, int passes, uint32_t* hist) {
    __shared__ uint32_t s_hist[kMaxPasses][kRadix];
    for (int i = threadIdx.x; i < kMaxPasses * kRadix; i += kSortThreads) (&s_hist[0][0])[i] = 0;
    __syncthreads();
    for (uint64_t i = (uint64_t)blockIdx.x * kSortThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kSortThreads) {
        uint32_t k = __ldg(keys + i) & mask;
        for (int p = 0; p < passes; ++p) atomicAdd(&s_hist[p][(k >> (8 * p)) & 0xffu], 1u);
    }
    __syncthreads();
    for (int p = 0; p < passes; ++p) {
        uint32_t c = s_hist[p][threadIdx.x];
        if (c) atomicAdd(hist + p * kRadix + threadIdx.x, c);
    }
}

struct PassArgs {
    const uint32_t* keys_in;
    const uint32_t* vals_in;
    uint32_t* keys_out;
    uint32_t* vals_out;
    uint32_t n;
    uint32_t mask;
    int shift;
    const uint32_t* hist;  // this pass's 256 bins
    uint32_t* lookback;    // [tiles][256]
    uint32_t* ticket;
    int* err;
};

__global__ void __launch_bounds__(kSortThreads, 4) sort_pass_kernel(const PassArgs a) {
    __shared__ uint32_t s_tile;
    __shared__ uint32_t s_warp_hist[kSortWarps][kRadix + 1];
    __shared__ uint32_t s_block_start[kRadix];
    __shared__ uint32_t s_global[kRadix];
    __shared__ uint32_t s_scan[kSortWarps + 1];
    __shared__ uint32_t s_keys[kSortTile];
    __shared__ uint32_t s_vals[kSortTile];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_tile = atomicAdd(a.ticket, 1u);
    for (int i = lane; i < kRadix + 1; i += 32) s_warp_hist[warp][i] = 0;
    __syncthreads();
    const uint32_t tile = s_tile;
    const uint64_t tile_base = (uint64_t)tile * kSortTile;
    const uint32_t tile_count = (uint32_t)min((uint64_t)kSortTile, (uint64_t)a.n - tile_base);

    // Warp-striped load: element index = tile_base + warp*512 + item*32 + lane.
    uint32_t key[kSortItems], val[kSortItems], rank[kSortItems];
    int dig[kSortItems];
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < kSortItems; ++i) {
        uint64_t idx = tile_base + (uint64_t)warp * (32 * kSortItems) + (uint64_t)i * 32 + lane;
        bool valid = idx < a.n;
        key[i] = valid ? __ldg(a.keys_in + idx) : 0u;
        val[i] = valid ? __ldg(a.vals_in + idx) : 0u;
        dig[i] = valid ? (int)(((key[i] & a.mask) >> a.shift) & 0xffu) : kRadix;
    }
    // Stable per-warp multi-split: items in order, lanes in order.
#pragma unroll
    for (int i = 0; i < kSortItems; ++i) {
        // lanes with the same digit: agree on validity and on each of the 8 bits
        uint32_t peers = __ballot_sync(0xffffffffu, dig[i] < kRadix);
        if (dig[i] >= kRadix) peers = ~peers;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const bool bit = (dig[i] >> b) & 1;
            const uint32_t bal = __ballot_sync(0xffffffffu, bit);
            peers &= bit ? bal : ~bal;
        }
        uint32_t before = peers & lt_mask;
        uint32_t base = s_warp_hist[warp][dig[i]];
        __syncwarp();
        if (before == 0) s_warp_hist[warp][dig[i]] = base + __popc(peers);
        __syncwarp();
        rank[i] = base + __popc(before);
    }
    __syncthreads();

    // Thread d owns digit d: warp prefix, block count, publish, look back.
    const int d = threadIdx.x;
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
        uint32_t c = s_warp_hist[w][d];
        s_warp_hist[w][d] = run;
        run += c;
    }
    const uint32_t block_count = run;
    uint32_t* lb = a.lookback + (size_t)tile * kRadix + d;
    if (tile == 0) st_relaxed_u32(lb, kLbIncl | block_count);
    else st_relaxed_u32(lb, kLbAgg | block_count);

    // Exclusive scans over digits: block-local starts and global bin starts.
    auto block_scan = [&](uint32_t v) -> uint32_t {
        uint32_t inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        if (lane == 31) s_scan[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            uint32_t wv = lane < kSortWarps ? s_scan[lane] : 0u;
            uint32_t wi = wv;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += t;
            }
            if (lane < kSortWarps) s_scan[lane] = wi - wv;
        }
        __syncthreads();
        uint32_t r = s_scan[warp] + inc - v;
        __syncthreads();
        return r;
    };
    s_block_start[d] = block_scan(block_count);
    const uint32_t global_bin = block_scan(__ldg(a.hist + d));

    uint32_t excl = 0;
    if (tile > 0) {
        int64_t pred = (int64_t)tile - 1;
        uint32_t spins = 0;
        while (pred >= 0) {
            uint32_t s = ld_relaxed_u32(a.lookback + (size_t)pred * kRadix + d);
            uint32_t flag = s & ~kLbMask;
            if (flag == 0) {
                if (++spins > kSpinLimit) {
                    set_error(a.err, kDevLookbackTimeout);
                    break;
                }
                __nanosleep(32);
                continue;
            }
            excl += s & kLbMask;
            if (flag == kLbIncl) break;
            --pred;
        }
        st_relaxed_u32(lb, kLbIncl | (excl + block_count));
    }
    s_global[d] = global_bin + excl;
    __syncthreads();

    // Stage in shared memory at the block-local sorted position.
#pragma unroll
    for (int i = 0; i < kSortItems; ++i) {
        if (dig[i] < kRadix) {
            uint32_t lp = s_block_start[dig[i]] + s_warp_hist[warp][dig[i]] + rank[i];
            s_keys[lp] = key[i];
            s_vals[lp] = val[i];
        }
    }
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < tile_count; j += kSortThreads) {
        uint32_t k = s_keys[j];
        uint32_t dj = ((k & a.mask) >> a.shift) & 0xffu;
        uint32_t pos = s_global[dj] + (j - s_block_start[dj]);
        if (pos < a.n) {
            a.keys_out[pos] = k;
            a.vals_out[pos] = s_vals[j];
        } else {
            set_error(a.err, kDevOutOfRange);
        }
    }
}

}  // namespace

bsx_status radix_sort_pairs(bsx_ctx* ctx, const uint32_t* d_keys, const uint32_t* d_vals, uint32_t n, uint32_t bits,
                            uint32_t* d_keys_out, uint32_t* d_vals_out) {
    if (n == 0) return BSX_OK;
    if (n >= (1u << 30)) return fail(ctx, BSX_ERR_CAPACITY, "radix sort supports fewer than 2^30 elements");
    uint32_t eff = (bits + 3u) / 4u * 4u;
    if (eff > 32) eff = 32;
    const uint32_t mask = eff >= 32 ? 0xffffffffu : ((1u << eff) - 1u);
    const int passes = (int)((eff + 7u) / 8u);
    if (passes == 0) {
        bsx_status s = check_cuda(ctx, cudaMemcpyAsync(d_keys_out, d_keys, (size_t)n * 4, cudaMemcpyDeviceToDevice, ctx->stream), "copy keys");
        if (s != BSX_OK) return s;
        return check_cuda(ctx, cudaMemcpyAsync(d_vals_out, d_vals, (size_t)n * 4, cudaMemcpyDeviceToDevice, ctx->stream), "copy values");
    }
    const uint32_t tiles = (n + kSortTile - 1) / kSortTile;
    bsx_status s = ensure(ctx, ctx->sort_tmp_k, (size_t)n * 4);
    if (s == BSX_OK) s = ensure(ctx, ctx->sort_tmp_v, (size_t)n * 4);
    if (s == BSX_OK) s = ensure(ctx, ctx->sort_hist, kMaxPasses * kRadix * 4);
    const size_t lb_words = (size_t)passes * tiles * kRadix + kMaxPasses;
    if (s == BSX_OK) s = ensure(ctx, ctx->sort_lookback, lb_words * 4);
    if (s != BSX_OK) return s;
    uint32_t* hist = ctx->sort_hist.as<uint32_t>();
    uint32_t* lookback = ctx->sort_lookback.as<uint32_t>();
    s = check_cuda(ctx, cudaMemsetAsync(hist, 0, kMaxPasses * kRadix * 4, ctx->stream), "memset histogram");
    if (s == BSX_OK) s = check_cuda(ctx, cudaMemsetAsync(lookback, 0, lb_words * 4, ctx->stream), "memset lookback");
    if (s != BSX_OK) return s;
    uint32_t hist_blocks = std::min<uint32_t>(tiles, 148u * 8u);
    prof_begin(ctx);
    sort_hist_kernel<<<hist_blocks, kSortThreads, 0, ctx->stream>>>(d_keys, n, mask, passes, hist);
    s = post_launch(ctx, "sort_hist_kernel");
    if (s != BSX_OK) return s;
    uint32_t* tmp_k = ctx->sort_tmp_k.as<uint32_t>();
    uint32_t* tmp_v = ctx->sort_tmp_v.as<uint32_t>();
    const uint32_t* src_k = d_keys;
    const uint32_t* src_v = d_vals;
    for (int p = 0; p < passes; ++p) {
        const bool to_out = ((passes - 1 - p) % 2) == 0;
        PassArgs a;
        a.keys_in = src_k;
        a.vals_in = src_v;
        a.keys_out = to_out ? d_keys_out : tmp_k;
        a.vals_out = to_out ? d_vals_out : tmp_v;
        a.n = n;
        a.mask = mask;
        a.shift = 8 * p;
        a.hist = hist + p * kRadix;
        a.lookback = lookback + (size_t)p * tiles * kRadix;
        a.ticket = lookback + (size_t)passes * tiles * kRadix + p;
        a.err = ctx->d_err;
        prof_begin(ctx);
        sort_pass_kernel<<<tiles, kSortThreads, 0, ctx->stream>>>(a);
        s = post_launch(ctx, "sort_pass_kernel");
        if (s != BSX_OK) return s;
        src_k = a.keys_out;
        src_v = a.vals_out;
    }
    return BSX_OK;
}

}  // namespace bsx

extern "C" bsx_status bsx_radix_argsort_u32(bsx_ctx* ctx, const uint32_t* d_keys, const uint32_t* d_values, uint32_t n,
                                            uint32_t sorting_bits, uint32_t* d_keys_out, uint32_t* d_values_out) {
    if (!ctx || (n && (!d_keys || !d_values || !d_keys_out || !d_values_out))) return BSX_ERR_INVALID_ARG;
    if (sorting_bits > 32) return bsx::fail(ctx, BSX_ERR_INVALID_ARG, "sorting_bits must be <= 32");
    if (n && (d_keys_out == d_keys || d_values_out == d_values))
        return bsx::fail(ctx, BSX_ERR_INVALID_ARG, "outputs must not alias inputs");
    cudaSetDevice(ctx->device);
    return bsx::radix_sort_pairs(ctx, d_keys, d_values, n, sorting_bits, d_keys_out, d_values_out);
}
