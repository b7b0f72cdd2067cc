// scan.cu - single-pass inclusive prefix sum with decoupled look-back.
//
// Replaces brush-prefix-sum's three-level Hillis-Steele scan
// (crates/brush-prefix-sum/src/lib.rs:11-87, kernels.rs:22-76) with one
// kernel: each 4096-element tile takes a ticket (so tiles wait only on tiles
// that are already running), reduces itself, publishes its aggregate, then
// warp 0 looks back over predecessors' published aggregates / inclusive
// prefixes (Merrill & Garland, "Single-pass Parallel Prefix Scan with
// Decoupled Look-back", 2016). Every wait is bounded: on expiry the tile
// records a device error and carries on, so the grid always terminates.
// Sums are u32 and wrap, as the reference's.
#include <mutex>

#include "common.cuh"
#include "lookback.cuh"

namespace bsx {

namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr uint32_t kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total to *total.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = warp_incl_scan(v);
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < (kScanThreads / 32) ? s_warp[lane] : 0u;
        uint32_t wi = warp_incl_scan(w);
        if (lane < (kScanThreads / 32)) s_warp[lane] = wi - w;
        if (lane == (kScanThreads / 32) - 1) s_warp[kScanThreads / 32] = wi;
    }
    __syncthreads();
    uint32_t excl = s_warp[warp] + incl - v;
    *total = s_warp[kScanThreads / 32];
    return excl;
}

}  // namespace

namespace {

__global__ void __launch_bounds__(kScanThreads) scan_kernel(const uint32_t* __restrict__ in,
                                                            const uint32_t* __restrict__ gather, uint32_t n,
                                                            uint32_t* __restrict__ out, uint64_t* status,
                                                            uint32_t* ticket, uint32_t* total_out, int* err,
                                                            int vec_in, int vec_out) {
    __shared__ uint32_t s_tile;
    __shared__ uint32_t s_warp[kScanThreads / 32 + 1];
    __shared__ uint32_t s_prefix;
    if (threadIdx.x == 0) s_tile = atomicAdd(ticket, 1u);
    __syncthreads();
    const uint32_t tile = s_tile;
    const uint64_t base = (uint64_t)tile * kScanTile + (uint64_t)threadIdx.x * kScanItems;
    uint32_t items[kScanItems];
    if (vec_in && !gather && base + kScanItems <= n) {
        const uint4* src = reinterpret_cast<const uint4*>(in + base);
#pragma unroll
        for (int q = 0; q < kScanItems / 4; ++q) {
            uint4 v = __ldg(src + q);
            items[4 * q] = v.x;
            items[4 * q + 1] = v.y;
            items[4 * q + 2] = v.z;
            items[4 * q + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            uint64_t i = base + k;
            items[k] = i < n ? (gather ? in[gather[i]] : in[i]) : 0u;
        }
    }
    uint32_t sum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) sum += items[k];
    uint32_t total;
    uint32_t excl = block_excl_scan(sum, s_warp, &total);
    if (threadIdx.x < 32) {
        uint32_t prefix = 0;
        if (tile == 0) {
            if (threadIdx.x == 0) st_relaxed_u64(status + tile, kFlagIncl | total);
        } else {
            if (threadIdx.x == 0) st_relaxed_u64(status + tile, kFlagAgg | total);
            prefix = lookback_exclusive(status, tile, err);
            if (threadIdx.x == 0) st_relaxed_u64(status + tile, kFlagIncl | (uint32_t)(prefix + total));
        }
        if (threadIdx.x == 0) {
            s_prefix = prefix;
            if (total_out && (uint64_t)(tile + 1) * kScanTile >= n) *total_out = prefix + total;
        }
    }
    __syncthreads();
    uint32_t run = s_prefix + excl;
    if (vec_out && base + kScanItems <= n) {
        uint4* dst = reinterpret_cast<uint4*>(out + base);
#pragma unroll
        for (int q = 0; q < kScanItems / 4; ++q) {
            uint4 v;
            run += items[4 * q];
            v.x = run;
            run += items[4 * q + 1];
            v.y = run;
            run += items[4 * q + 2];
            v.z = run;
            run += items[4 * q + 3];
            v.w = run;
            dst[q] = v;
        }
    } else {
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            run += items[k];
            if (base + k < n) out[base + k] = run;
        }
    }
}

}  // namespace

size_t scan_status_words(uint32_t n_tiles) { return (size_t)n_tiles + 2; }

bsx_status scan_inclusive_u32(bsx_ctx* ctx, const uint32_t* d_in, const uint32_t* d_gather, uint32_t n,
                              uint32_t* d_out, uint32_t* d_total) {
    if (n == 0) {
        if (d_total) return check_cuda(ctx, cudaMemsetAsync(d_total, 0, 4, ctx->stream), "memset total");
        return BSX_OK;
    }
    const uint32_t tiles = (uint32_t)(((uint64_t)n + kScanTile - 1) / kScanTile);
    bsx_status s = ensure(ctx, ctx->scan_status, scan_status_words(tiles) * sizeof(uint64_t));
    if (s != BSX_OK) return s;
    uint64_t* status = ctx->scan_status.as<uint64_t>();
    s = check_cuda(ctx, cudaMemsetAsync(status, 0, scan_status_words(tiles) * sizeof(uint64_t), ctx->stream),
                   "memset scan status");
    if (s != BSX_OK) return s;
    uint32_t* ticket = reinterpret_cast<uint32_t*>(status + tiles);
    const int vec_in = ((uintptr_t)d_in % 16) == 0;
    const int vec_out = ((uintptr_t)d_out % 16) == 0;
    prof_begin(ctx);
    scan_kernel<<<tiles, kScanThreads, 0, ctx->stream>>>(d_in, d_gather, n, d_out, status, ticket, d_total,
                                                           ctx->d_err, vec_in, vec_out);
    return post_launch(ctx, "scan_kernel");
}

}  // namespace bsx

extern "C" bsx_status bsx_prefix_sum_u32(bsx_ctx* ctx, const uint32_t* d_in, uint32_t n, uint32_t* d_out) {
    if (!ctx || (n && (!d_in || !d_out))) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    return bsx::scan_inclusive_u32(ctx, d_in, nullptr, n, d_out, nullptr);
}

// ---------------------------------------------------------------------------
// Allocation-free prefix sum.
//
// For callers that must not allocate GPU memory: code running inside a
// memory pool or arena that forbids foreign allocations, real-time loops
// where cudaMalloc's implicit device synchronisation is unacceptable, and
// plugin hosts that do not let a plugin create a bsx context (creating one
// allocates its error word and pinned readback slots). The look-back state
// of this scan lives in a fixed file-scope device array instead of a
// context workspace, so a call enqueues one memset and one kernel and
// allocates nothing.
//
// Limits and rules:
//  - n <= BSX_PREFIX_SUM_NOALLOC_MAX_N (16,769,024); larger n is rejected.
//  - The array is one per GPU that loads this library and stays resident
//    until the process exits (32 KiB).
//  - Every call shares the array, so calls whose execution overlaps on the
//    GPU (different streams, or different host threads on the same device)
//    race and produce wrong results; serialise them.
//  - The stream must belong to the current device (another device's stream
//    is rejected with BSX_ERR_INVALID_ARG); the null stream means the
//    current device's default stream.
//  - The first call on a device looks up the array's device address (with
//    that device current); make that first call before any stream capture.
//  - Device-side look-back waits are bounded; a timed-out wait is not
//    reported by this entry point (it has no context to report into).
// ---------------------------------------------------------------------------
namespace {

constexpr uint32_t kNoAllocTiles = 4094;  // 4094 * 4096 = 16,769,024 elements
static __device__ __align__(256) uint64_t g_noalloc_scan_state[kNoAllocTiles + 2];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256];  // device address of g_noalloc_scan_state, per device ordinal

}  // namespace

extern "C" bsx_status bsx_prefix_sum_u32_noalloc(const uint32_t* d_in, uint32_t n, uint32_t* d_out,
                                                 void* cuda_stream) {
    static_assert((uint64_t)kNoAllocTiles * bsx::kScanTile == BSX_PREFIX_SUM_NOALLOC_MAX_N, "limit mismatch");
    if (n && (!d_in || !d_out)) return BSX_ERR_INVALID_ARG;
    if (n > BSX_PREFIX_SUM_NOALLOC_MAX_N) return BSX_ERR_CAPACITY;
    if (n == 0) return BSX_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return BSX_ERR_CUDA;
    cudaStream_t stream = (cudaStream_t)cuda_stream;
    // The scratch address below is the current device's copy of the array, so
    // a stream of another device would run the scan against the wrong memory.
    if (stream) {
        int stream_dev = -1;
        if (cudaStreamGetDevice(stream, &stream_dev) != cudaSuccess) return BSX_ERR_CUDA;
        if (stream_dev != dev) return BSX_ERR_INVALID_ARG;
    }
    void* state = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            // Host code cannot use the array's name as a device address; ask the
            // runtime for this device's copy (the current device is `dev`).
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_scan_state) != cudaSuccess || !p) return BSX_ERR_CUDA;
            g_noalloc_ptr[dev] = p;
        }
        state = g_noalloc_ptr[dev];
    }
    const uint32_t tiles = (uint32_t)(((uint64_t)n + bsx::kScanTile - 1) / bsx::kScanTile);
    uint64_t* status = static_cast<uint64_t*>(state);
    // The look-back words and the ticket must start at zero on every call.
    if (cudaMemsetAsync(status, 0, bsx::scan_status_words(tiles) * sizeof(uint64_t), stream) != cudaSuccess)
        return BSX_ERR_CUDA;
    uint32_t* ticket = reinterpret_cast<uint32_t*>(status + tiles);
    const int vec_in = ((uintptr_t)d_in % 16) == 0;
    const int vec_out = ((uintptr_t)d_out % 16) == 0;
    // cudaLaunchKernel reports this launch's own error; an error left by the
    // caller's earlier CUDA calls is neither reported here nor cleared.
    const uint32_t* gather = nullptr;
    uint32_t* total = nullptr;
    int* err = nullptr;
    void* args[] = {(void*)&d_in, (void*)&gather, (void*)&n,      (void*)&d_out,  (void*)&status,
                    (void*)&ticket, (void*)&total, (void*)&err, (void*)&vec_in, (void*)&vec_out};
    const cudaError_t e = cudaLaunchKernel((const void*)bsx::scan_kernel, dim3(tiles), dim3(bsx::kScanThreads), args,
                                           0, stream);
    return e == cudaSuccess ? BSX_OK : BSX_ERR_CUDA;
}
