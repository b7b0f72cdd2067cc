// emit.cu - intersection emission and per-tile ranges.
//
// emit_kernel restates map_gaussians_to_intersect_kernel
// (crates/brush-render/src/kernels/map_gaussians.rs:14-92): one thread per
// visible splat in depth order walks its tile bbox row-major, writes
// (tile id, splat id) for every tile passing the StopThePop test into the
// slots reserved by the inclusive count scan, and pads any shortfall with the
// sentinel tile id T (sorted after every real tile). The splat id written is
// the global id (projected rows are global-id indexed here).
//
// tile_offsets_kernel restates get_tile_offsets
// (crates/brush-render/src/get_tile_offset.rs:10-62).
#include "splat_math.cuh"

namespace bsx {

namespace {

__global__ void __launch_bounds__(256) emit_kernel(const float* __restrict__ projected,
                                                   const uint32_t* __restrict__ depth_order,
                                                   const uint32_t* __restrict__ cum, uint32_t num_visible,
                                                   uint32_t tbw, uint32_t tbh, uint32_t* __restrict__ tile_out,
                                                   uint32_t* __restrict__ gid_out, uint32_t num_isect, int* err) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= num_visible) return;
    const uint32_t g = __ldg(depth_order + i);
    const float4* row = reinterpret_cast<const float4*>(projected + (size_t)g * BSX_PROJECTED_LANES);
    const float4 r0 = __ldg(row), r1 = __ldg(row + 1), r2 = __ldg(row + 2);
    const float x = r0.x, y = r0.y;
    const S2 conic{r0.z, r0.w, r1.x};
    // ln(255 * opacity): the projection pass stored it from the same opacity.
    const float pt = r2.z;
    float ex, ey;
    bbox_extent(conic, pt, &ex, &ey);
    const TileBox bb = tile_bbox(x, y, ex, ey, tbw, tbh);
    const uint32_t base = i == 0 ? 0u : __ldg(cum + i - 1);
    const uint32_t budget = __ldg(cum + i) - base;
    if (base > num_isect || budget > num_isect - base) {
        set_error(err, kDevOutOfRange);
        return;
    }
    uint32_t hit = 0;
    for (uint32_t ty = bb.min_y; ty < bb.max_y && hit < budget; ++ty)
        for (uint32_t tx = bb.min_x; tx < bb.max_x && hit < budget; ++tx)
            if (tile_contrib(tx, ty, x, y, conic, pt)) {
                tile_out[base + hit] = tx + ty * tbw;
                gid_out[base + hit] = g;
                ++hit;
            }
    const uint32_t sentinel = tbw * tbh;
    for (uint32_t k = hit; k < budget; ++k) {
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

}  // namespace

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
