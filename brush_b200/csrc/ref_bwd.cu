// ref_bwd.cu - the backward operators with the reference's own signatures.
//
// SplatBwdOps::rasterize_bwd / rasterize_bwd_with_refine_weight / project_bwd
// (crates/brush-render-bwd/src/burn_glue.rs:80-141) are stateless and work on
// compact-indexed tensors: projected rows [V,10] and the gradient rows
// v_combined [V,11] are indexed by the depth rank of a visible splat
// (compact id), the intersection list holds compact ids, and
// global_from_compact_gid [V] maps a compact id to the splat row of the dense
// outputs. This library's pipeline indexes the same rows by global id, with
// 12-lane rows (three 16-byte words) so that the rasterizers stage them with
// vector loads and accumulate gradients with vector atomics.
//
// These entry points adapt the reference layout to the same kernels the
// training step runs:
//   rasterize: [V,10] rows -> 12-lane rows (lane 10 = ln(255 opacity), the
//   raster pre-filter threshold, recomputed exactly as the projection writes
//   it) -> raster backward over the caller's intersection list and shortened
//   tile ranges -> the 11 reference lanes of each row.
//   project: [V,11] rows scattered to dense 12-lane rows by
//   global_from_compact_gid -> projection backward over all N splats.
// The callers' tensors are not trusted: an intersection id >= V, a tile range
// outside [0, M] or a global id >= N is skipped (as the reference's checked
// launches skip out-of-bounds accesses) and reported as BSX_ERR_INVALID_ARG
// by the next bsx_sync.
#include "common.cuh"

namespace bsx {

bsx_status launch_raster_bwd(bsx_ctx* ctx, const uint32_t* isect_gid, const uint32_t* tile_offsets,
                             const float* projected, const float* image, const float* v_output, float* v_grad,
                             const uint8_t* isect_mask, const uint32_t* order, const bsx_project_uniforms& u,
                             const float bg[3], int smooth, int refine);
bsx_status launch_project_bwd(bsx_ctx* ctx, const bsx_project_uniforms& uni, const float* transforms, const float* sh,
                              const float* raw_opac, uint32_t n, uint32_t coeffs, int degree, int mip,
                              const float* v_grad, float* v_transforms, float* v_sh, float* v_opac, float* v_refine,
                              const FusedAdam* adam, const GradPush* push = nullptr);

namespace {

constexpr int kRefThreads = 256;

uint32_t ref_blocks(uint64_t items) {
    const uint64_t b = (items + kRefThreads - 1) / kRefThreads;
    return (uint32_t)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

// [V,10] reference rows -> [V+1,12] rows; row V is a splat that nothing can
// accept (zero opacity, pre-filter threshold -inf), the target of skipped ids.
__global__ void __launch_bounds__(kRefThreads)
    widen_rows_kernel(const float* __restrict__ rows10, uint32_t v, float4* __restrict__ rows12) {
    for (uint32_t c = blockIdx.x * kRefThreads + threadIdx.x; c <= v; c += gridDim.x * kRefThreads) {
        if (c == v) {
            rows12[3 * (size_t)c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            rows12[3 * (size_t)c + 1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            rows12[3 * (size_t)c + 2] = make_float4(0.0f, 0.0f, -INFINITY, 0.0f);
            continue;
        }
        const float* r = rows10 + (size_t)c * 10;
        float x[10];
#pragma unroll
        for (int k = 0; k < 10; ++k) x[k] = __ldg(r + k);
        // the projection writes ln(255 o) for every visible row (o >= 1/255 there)
        const float pt = bsx_logf(x[5] * 255.0f);
        rows12[3 * (size_t)c] = make_float4(x[0], x[1], x[2], x[3]);
        rows12[3 * (size_t)c + 1] = make_float4(x[4], x[5], x[6], x[7]);
        rows12[3 * (size_t)c + 2] = make_float4(x[8], x[9], pt, 0.0f);
    }
}

// Intersection ids and tile ranges, bounds-checked: ids >= V map to the inert
// row V; each range is clamped into [0, M] with end >= start.
__global__ void __launch_bounds__(kRefThreads)
    check_isects_kernel(const uint32_t* __restrict__ ids_in, uint32_t m, uint32_t v, const uint32_t* __restrict__ off_in,
                        uint32_t tiles, uint32_t* __restrict__ ids_out, uint32_t* __restrict__ off_out, int* err) {
    const uint32_t stride = gridDim.x * kRefThreads;
    for (uint32_t i = blockIdx.x * kRefThreads + threadIdx.x; i < m; i += stride) {
        const uint32_t id = __ldg(ids_in + i);
        if (id >= v) set_error(err, kDevBadIndex);
        ids_out[i] = id < v ? id : v;
    }
    for (uint32_t t = blockIdx.x * kRefThreads + threadIdx.x; t < tiles; t += stride) {
        const uint32_t lo = __ldg(off_in + 2 * t), hi = __ldg(off_in + 2 * t + 1);
        if (lo > m || hi > m) set_error(err, kDevBadIndex);
        const uint32_t l = min(lo, m);
        off_out[2 * t] = l;
        off_out[2 * t + 1] = max(min(hi, m), l);
    }
}

// 12-lane gradient rows -> the 11 reference lanes (xy, conic, rgb, alpha, refine, depth).
__global__ void __launch_bounds__(kRefThreads)
    narrow_grads_kernel(const float* __restrict__ g12, uint32_t v, float* __restrict__ g11) {
    const uint64_t total = (uint64_t)v * BSX_COMPACT_GRAD_LANES;
    for (uint64_t e = (uint64_t)blockIdx.x * kRefThreads + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * kRefThreads) {
        const uint64_t row = e / BSX_COMPACT_GRAD_LANES, lane = e % BSX_COMPACT_GRAD_LANES;
        g11[e] = g12[row * kGradStride + lane];
    }
}

// [V,11] compact rows -> dense [N,12] rows at global_from_compact_gid (zeroed before).
__global__ void __launch_bounds__(kRefThreads)
    scatter_grads_kernel(const float* __restrict__ g11, const uint32_t* __restrict__ gid, uint32_t v, uint32_t n,
                         float* __restrict__ g12, int* err) {
    for (uint32_t c = blockIdx.x * kRefThreads + threadIdx.x; c < v; c += gridDim.x * kRefThreads) {
        const uint32_t g = __ldg(gid + c);
        if (g >= n) {
            set_error(err, kDevBadIndex);
            continue;
        }
        const float* src = g11 + (size_t)c * BSX_COMPACT_GRAD_LANES;
        float* dst = g12 + (size_t)g * kGradStride;
#pragma unroll
        for (int k = 0; k < BSX_COMPACT_GRAD_LANES; ++k) dst[k] = __ldg(src + k);
    }
}

int degree_of(uint32_t c) {
    for (int d = 0; d <= 4; ++d)
        if ((uint32_t)((d + 1) * (d + 1)) == c) return d;
    return -1;
}

}  // namespace

}  // namespace bsx

using namespace bsx;

extern "C" {

bsx_status bsx_rasterize_bwd_ref(bsx_ctx* ctx, const float* d_out_img, const float* d_projected, uint32_t num_visible,
                                 const uint32_t* d_compact_gid_from_isect, uint32_t num_intersections,
                                 const uint32_t* d_tile_offsets, const float background[3], uint32_t img_w,
                                 uint32_t img_h, const float* d_v_output, int32_t smooth_cutoff,
                                 int32_t compute_refine_weight, int32_t render_depth, float* d_v_combined) {
    if (!ctx || !background || !d_out_img || !d_v_output || !d_tile_offsets) return BSX_ERR_INVALID_ARG;
    if (num_visible && (!d_projected || !d_v_combined)) return BSX_ERR_INVALID_ARG;
    if (num_intersections && !d_compact_gid_from_isect) return BSX_ERR_INVALID_ARG;
    if (render_depth) return fail(ctx, BSX_ERR_UNSUPPORTED, "depth rendering (RgbaAndDepth) is not built");
    if (img_w == 0 || img_h == 0 || img_w > 16384 || img_h > 16384)
        return fail(ctx, BSX_ERR_INVALID_ARG, "image size out of range");
    if (((uintptr_t)d_out_img | (uintptr_t)d_v_output) % 16)
        return fail(ctx, BSX_ERR_INVALID_ARG, "out_img and v_output must be 16-byte aligned");
    if (num_intersections >= (1u << 30)) return fail(ctx, BSX_ERR_CAPACITY, "intersection count out of range");
    cudaSetDevice(ctx->device);
    const uint32_t v = num_visible, m = num_intersections;
    if (v == 0) return BSX_OK;
    bsx_status s = check_cuda(ctx, cudaMemsetAsync(d_v_combined, 0, (size_t)v * BSX_COMPACT_GRAD_LANES * 4, ctx->stream),
                              "memset v_combined");
    if (s != BSX_OK || m == 0) return s;
    bsx_project_uniforms u{};
    u.img_w = img_w;
    u.img_h = img_h;
    u.tile_bw = (img_w + kTile - 1) / kTile;
    u.tile_bh = (img_h + kTile - 1) / kTile;
    const uint32_t tiles = u.tile_bw * u.tile_bh;
    if ((s = ensure(ctx, ctx->ref_rows, ((size_t)v + 1) * BSX_PROJECTED_LANES * 4)) != BSX_OK) return s;
    if ((s = ensure(ctx, ctx->ref_grad, ((size_t)v + 1) * kGradStride * 4)) != BSX_OK) return s;
    if ((s = ensure(ctx, ctx->ref_ids, (size_t)m * 4)) != BSX_OK) return s;
    if ((s = ensure(ctx, ctx->ref_offsets, (size_t)tiles * 8)) != BSX_OK) return s;
    prof_begin(ctx);
    widen_rows_kernel<<<ref_blocks((uint64_t)v + 1), kRefThreads, 0, ctx->stream>>>(d_projected, v,
                                                                                  ctx->ref_rows.as<float4>());
    if ((s = post_launch(ctx, "widen_rows_kernel")) != BSX_OK) return s;
    prof_begin(ctx);
    check_isects_kernel<<<ref_blocks(m > tiles ? m : tiles), kRefThreads, 0, ctx->stream>>>(
        d_compact_gid_from_isect, m, v, d_tile_offsets, tiles, ctx->ref_ids.as<uint32_t>(),
        ctx->ref_offsets.as<uint32_t>(), ctx->d_err);
    if ((s = post_launch(ctx, "check_isects_kernel")) != BSX_OK) return s;
    s = check_cuda(ctx, cudaMemsetAsync(ctx->ref_grad.p, 0, ((size_t)v + 1) * kGradStride * 4, ctx->stream),
                   "memset gradient rows");
    if (s != BSX_OK) return s;
    s = launch_raster_bwd(ctx, ctx->ref_ids.as<uint32_t>(), ctx->ref_offsets.as<uint32_t>(), ctx->ref_rows.as<float>(),
                          d_out_img, d_v_output, ctx->ref_grad.as<float>(), nullptr, nullptr, u, background,
                          smooth_cutoff != 0,
                          compute_refine_weight != 0);
    if (s != BSX_OK) return s;
    prof_begin(ctx);
    narrow_grads_kernel<<<ref_blocks((uint64_t)v * BSX_COMPACT_GRAD_LANES), kRefThreads, 0, ctx->stream>>>(
        ctx->ref_grad.as<float>(), v, d_v_combined);
    return post_launch(ctx, "narrow_grads_kernel");
}

bsx_status bsx_project_bwd_ref(bsx_ctx* ctx, const float* d_transforms, const float* d_sh_coeffs,
                               const float* d_raw_opac, uint32_t num_splats, uint32_t sh_coeffs_per_splat,
                               const uint32_t* d_global_from_compact_gid, uint32_t num_visible,
                               const bsx_project_uniforms* uniforms, int32_t render_mode, const float* d_v_combined,
                               float* d_v_transforms, float* d_v_sh_coeffs, float* d_v_raw_opac,
                               float* d_v_refine_weight) {
    if (!ctx || !uniforms) return BSX_ERR_INVALID_ARG;
    const uint32_t n = num_splats, v = num_visible;
    if (n && (!d_transforms || !d_sh_coeffs || !d_raw_opac || !d_v_transforms || !d_v_sh_coeffs || !d_v_raw_opac ||
              !d_v_refine_weight))
        return BSX_ERR_INVALID_ARG;
    if (v && (!d_global_from_compact_gid || !d_v_combined)) return BSX_ERR_INVALID_ARG;
    if (render_mode != BSX_RENDER_DEFAULT && render_mode != BSX_RENDER_MIP)
        return fail(ctx, BSX_ERR_INVALID_ARG, "render_mode");
    const int degree = degree_of(sh_coeffs_per_splat);
    if (degree < 0) return fail(ctx, BSX_ERR_SHAPE, "sh_coeffs must be [N, (degree+1)^2, 3] with degree <= 4");
    if ((uint32_t)degree != uniforms->sh_degree)
        return fail(ctx, BSX_ERR_SHAPE, "project uniforms name another SH degree than sh_coeffs");
    if (v > n) return fail(ctx, BSX_ERR_SHAPE, "more visible splats than splats");
    if (((uintptr_t)d_sh_coeffs | (uintptr_t)d_raw_opac) % 4 || (uintptr_t)d_transforms % 8)
        return fail(ctx, BSX_ERR_INVALID_ARG, "transforms must be 8-byte aligned, sh / opacities 4-byte aligned");
    if (n == 0) return BSX_OK;
    cudaSetDevice(ctx->device);
    bsx_status s = ensure(ctx, ctx->ref_grad, (size_t)n * kGradStride * 4);
    if (s != BSX_OK) return s;
    s = check_cuda(ctx, cudaMemsetAsync(ctx->ref_grad.p, 0, (size_t)n * kGradStride * 4, ctx->stream),
                   "memset gradient rows");
    if (s != BSX_OK) return s;
    if (v) {
        prof_begin(ctx);
        scatter_grads_kernel<<<ref_blocks(v), kRefThreads, 0, ctx->stream>>>(
            d_v_combined, d_global_from_compact_gid, v, n, ctx->ref_grad.as<float>(), ctx->d_err);
        if ((s = post_launch(ctx, "scatter_grads_kernel")) != BSX_OK) return s;
    }
    bsx_project_uniforms u = *uniforms;
    u.total_splats = n;
    return launch_project_bwd(ctx, u, d_transforms, d_sh_coeffs, d_raw_opac, n, sh_coeffs_per_splat, degree,
                              render_mode == BSX_RENDER_MIP, ctx->ref_grad.as<float>(), d_v_transforms, d_v_sh_coeffs,
                              d_v_raw_opac, d_v_refine_weight, nullptr);
}

}  // extern "C"
