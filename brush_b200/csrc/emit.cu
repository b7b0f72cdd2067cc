// emit.cu - intersection emission and per-tile ranges.
//
// emit_kernel restates map_gaussians_to_intersect_kernel
// (crates/brush-render/src/kernels/map_gaussians.rs:14-92): for every visible
// splat in depth order, the tiles of its bbox in row-major order that pass
// the StopThePop test are written as (tile id, splat id) into the slots
// reserved by the inclusive count scan, and any shortfall is padded with the
// sentinel tile id T (sorted after every real tile). A warp walks its 32
// splats' boxes together (tile_walk.cuh). The splat id written is the global
// id (projected rows are global-id indexed here).
//
// tile_offsets_kernel restates get_tile_offsets
// (crates/brush-render/src/get_tile_offset.rs:10-62).
#include "tile_walk.cuh"

namespace bsx {

namespace {

__global__ void __launch_bounds__(256) emit_kernel(const float* __restrict__ projected,
                                                   const uint32_t* __restrict__ depth_order,
                                                   const uint32_t* __restrict__ cum, uint32_t num_visible,
                                                   uint32_t tbw, uint32_t tbh, uint32_t* __restrict__ tile_out,
                                                   uint32_t* __restrict__ gid_out, uint32_t num_isect, int* err) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    WalkSplat ws{0u, 0u, 0u, 0u, 0.0f, 0.0f, S2{0.0f, 0.0f, 0.0f}, 0.0f};
    uint32_t g = 0, base = 0, budget = 0;
    if (i < num_visible) {
        g = __ldg(depth_order + i);
        const float4* row = reinterpret_cast<const float4*>(projected + (size_t)g * BSX_PROJECTED_LANES);
        const float4 r0 = __ldg(row), r1 = __ldg(row + 1), r2 = __ldg(row + 2);
        const S2 conic{r0.z, r0.w, r1.x};
        // ln(255 * opacity): the projection pass stored it from the same opacity.
        const float pt = r2.z;
        float ex, ey;
        bbox_extent(conic, pt, &ex, &ey);
        const TileBox bb = tile_bbox(r0.x, r0.y, ex, ey, tbw, tbh);
        base = i == 0 ? 0u : __ldg(cum + i - 1);
        budget = __ldg(cum + i) - base;
        if (base > num_isect || budget > num_isect - base) {
            set_error(err, kDevOutOfRange);
            budget = 0;
        } else {
            const uint32_t bw = bb.max_x > bb.min_x ? bb.max_x - bb.min_x : 0u;
            const uint32_t bh = bb.max_y > bb.min_y ? bb.max_y - bb.min_y : 0u;
            ws = WalkSplat{bb.min_x, bb.min_y, bw, bw * bh, r0.x, r0.y, conic, pt};
        }
    }
    // Hits of one splat land at consecutive slots from its scan offset, in
    // row-major box order; a warp iteration writes one contiguous run.
    uint32_t written = 0;
    warp_tile_walk(ws, [&](const WalkStep& s) {
        const uint32_t o_written = __shfl_sync(kFullMask, written, s.owner);
        const uint32_t o_base = __shfl_sync(kFullMask, base, s.owner);
        const uint32_t o_budget = __shfl_sync(kFullMask, budget, s.owner);
        const uint32_t o_gid = __shfl_sync(kFullMask, g, s.owner);
        const uint32_t slot = o_written + s.before;
        if (s.hit && slot < o_budget) {
            tile_out[o_base + slot] = s.tx + s.ty * tbw;
            gid_out[o_base + slot] = o_gid;
        }
        written += s.own;
    });
    // pad any shortfall with the sentinel tile id (sorted after every real tile)
    const uint32_t sentinel = tbw * tbh;
    for (uint32_t k = written; k < budget; ++k) {
        tile_out[base + k] = sentinel;
        gid_out[base + k] = g;
    }
}

constexpr uint32_t kChecksPerThread = 8;

__global__ void __launch_bounds__(256) tile_offsets_kernel(const uint32_t* __restrict__ ids, uint32_t n,
                                                           uint32_t num_tiles, uint32_t* __restrict__ off) {
    const uint64_t base = (uint64_t)blockIdx.x * blockDim.x * kChecksPerThread + threadIdx.x;
#pragma unroll
    for (uint32_t c = 0; c < kChecksPerThread; ++c) {
        const uint64_t k = base + (uint64_t)c * blockDim.x;
        if (k >= n) break;
        const uint32_t tid = __ldg(ids + k);
        if (k == 0) {
            if (tid < num_tiles) off[tid * 2] = 0;
        } else {
            const uint32_t prev = __ldg(ids + k - 1);
            if (tid != prev) {
                if (prev < num_tiles) off[prev * 2 + 1] = (uint32_t)k;
                if (tid < num_tiles) off[tid * 2] = (uint32_t)k;
            }
        }
        if (k == n - 1 && tid < num_tiles) off[tid * 2 + 1] = (uint32_t)(k + 1);
    }
}

// Launch order of the tiles for the rasterizers: by descending intersection
// count, so the longest tiles start first and the short ones fill the tail
// (in tile order, clustered scenes leave long tiles running alone at the end).
// A counting sort into 256 buckets of count >> shift (shift fits the largest
// count into 8 bits); the order within a bucket is arbitrary, which no output
// depends on (tiles are independent). One block; each pass over the tile
// ranges loads kOrderPer tiles per thread at once (one memory round trip per
// 8192 tiles instead of one per tile and thread).
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 256;
constexpr int kOrderPer = 8;

__global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(const uint32_t* __restrict__ off, uint32_t num_tiles,
                                                                   uint32_t* __restrict__ order) {
    __shared__ uint32_t s_cur[kOrderBuckets];
    __shared__ uint32_t s_max;
    if (threadIdx.x < kOrderBuckets) s_cur[threadIdx.x] = 0;
    if (threadIdx.x == 0) s_max = 0;
    __syncthreads();
    // fn(t, count) for every tile, kOrderPer independent loads per thread per round
    auto for_tiles = [&](auto fn) {
        for (uint32_t base = 0; base < num_tiles; base += kOrderThreads * kOrderPer) {
            uint2 r[kOrderPer];
#pragma unroll
            for (int k = 0; k < kOrderPer; ++k) {
                const uint32_t t = base + k * kOrderThreads + threadIdx.x;
                r[k] = t < num_tiles ? __ldg(reinterpret_cast<const uint2*>(off) + t) : make_uint2(0u, 0u);
            }
#pragma unroll
            for (int k = 0; k < kOrderPer; ++k) {
                const uint32_t t = base + k * kOrderThreads + threadIdx.x;
                if (t < num_tiles) fn(t, r[k].y > r[k].x ? r[k].y - r[k].x : 0u);
            }
        }
    };
    uint32_t m = 0;
    for_tiles([&](uint32_t, uint32_t c) { m = max(m, c); });
    for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(&s_max, m);
    __syncthreads();
    const uint32_t shift = s_max >= (uint32_t)kOrderBuckets ? 32 - __clz(s_max) - 8 : 0;
    auto bucket = [&](uint32_t c) { return (uint32_t)(kOrderBuckets - 1) - (c >> shift); };
    for_tiles([&](uint32_t, uint32_t c) { atomicAdd(&s_cur[bucket(c)], 1u); });
    __syncthreads();
    // exclusive prefix over the buckets (Hillis-Steele on the first 256 threads)
    uint32_t v = threadIdx.x < kOrderBuckets ? s_cur[threadIdx.x] : 0u;
    const uint32_t own = v;
    for (int d = 1; d < kOrderBuckets; d <<= 1) {
        const uint32_t add = (threadIdx.x < kOrderBuckets && (int)threadIdx.x >= d) ? s_cur[threadIdx.x - d] : 0u;
        __syncthreads();
        v += add;
        if (threadIdx.x < kOrderBuckets) s_cur[threadIdx.x] = v;
        __syncthreads();
    }
    if (threadIdx.x < kOrderBuckets) s_cur[threadIdx.x] = v - own;
    __syncthreads();
    for_tiles([&](uint32_t t, uint32_t c) { order[atomicAdd(&s_cur[bucket(c)], 1u)] = t; });
}

}  // namespace

bsx_status tile_order(bsx_ctx* ctx, const uint32_t* d_off, uint32_t num_tiles, uint32_t* d_order) {
    if (num_tiles == 0) return BSX_OK;
    prof_begin(ctx);
    tile_order_kernel<<<1, kOrderThreads, 0, ctx->stream>>>(d_off, num_tiles, d_order);
    return post_launch(ctx, "tile_order_kernel");
}

bsx_status launch_emit(bsx_ctx* ctx, const float* projected, const uint32_t* depth_order, const uint32_t* cum,
                       uint32_t num_visible, uint32_t tbw, uint32_t tbh, uint32_t* tile_out, uint32_t* gid_out,
                       uint32_t num_isect) {
    if (num_visible == 0) return BSX_OK;
    prof_begin(ctx);
    emit_kernel<<<(num_visible + 255) / 256, 256, 0, ctx->stream>>>(projected, depth_order, cum, num_visible, tbw,
                                                                    tbh, tile_out, gid_out, num_isect, ctx->d_err);
    return post_launch(ctx, "emit_kernel");
}

bsx_status tile_offsets(bsx_ctx* ctx, const uint32_t* d_ids, uint32_t n, uint32_t num_tiles, uint32_t* d_off) {
    bsx_status s = check_cuda(ctx, cudaMemsetAsync(d_off, 0, (size_t)num_tiles * 2 * 4, ctx->stream), "memset tile offsets");
    if (s != BSX_OK || n == 0) return s;
    const uint32_t per_block = 256 * kChecksPerThread;
    prof_begin(ctx);
    tile_offsets_kernel<<<(n + per_block - 1) / per_block, 256, 0, ctx->stream>>>(d_ids, n, num_tiles, d_off);
    return post_launch(ctx, "tile_offsets_kernel");
}

}  // namespace bsx

extern "C" bsx_status bsx_get_tile_offsets(bsx_ctx* ctx, const uint32_t* d_tile_ids, uint32_t n, uint32_t num_tiles,
                                           uint32_t* d_offsets) {
    if (!ctx || !d_offsets || (n && !d_tile_ids)) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    return bsx::tile_offsets(ctx, d_tile_ids, n, num_tiles, d_offsets);
}
