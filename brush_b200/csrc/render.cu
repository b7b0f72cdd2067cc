// render.cu - host orchestration of the forward render and the backward
// entry points (the SplatOps / SplatBwdOps boundary).
//
// Forward order (crates/brush-render/src/render.rs:78-543):
//   project+SH+compaction -> one readback of (visible, intersections)
//   -> stable depth sort of visible ids -> inclusive scan of their tile
//   counts in depth order -> intersection emission -> stable tile sort
//   -> per-tile ranges -> rasterize.
// Ties in depth are broken by global id (the reference's order there depends
// on atomic scheduling).
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace bsx {
bsx_status launch_project_fwd(bsx_ctx* ctx, const bsx_project_uniforms& uni, const float* transforms,
                              const float* sh, const float* raw_opac, uint32_t n, uint32_t coeffs, int degree,
                              int mip, float* projected, uint32_t* counts, float* max_radius, uint32_t* vis_gid,
                              uint32_t* depth_key, uint32_t* scalars, uint32_t* vis_mask, uint32_t* depth_dense);
bsx_status launch_emit(bsx_ctx* ctx, const float* projected, const uint32_t* depth_order, const uint32_t* cum,
                       uint32_t num_visible, uint32_t tbw, uint32_t tbh, uint32_t* tile_out, uint32_t* gid_out,
                       uint32_t num_isect);
bsx_status launch_raster_fwd(bsx_ctx* ctx, const uint32_t* isect_gid, uint32_t* tile_offsets, const float* projected,
                             float* image, uint32_t* image_packed, float* visible, uint8_t* isect_mask,
                             const bsx_project_uniforms& u, const float bg[3], int bwd_info, int smooth);
bsx_status launch_raster_bwd(bsx_ctx* ctx, const uint32_t* isect_gid, const uint32_t* tile_offsets,
                             const float* projected, const float* image, const float* v_output, float* v_grad,
                             const uint8_t* isect_mask, const uint32_t* order, const bsx_project_uniforms& u,
                             const float bg[3], int smooth, int refine);
bsx_status launch_project_bwd(bsx_ctx* ctx, const bsx_project_uniforms& uni, const float* transforms, const float* sh,
                              const float* raw_opac, uint32_t n, uint32_t coeffs, int degree, int mip,
                              const float* v_grad, float* v_transforms, float* v_sh, float* v_opac, float* v_refine,
                              const FusedAdam* adam, const GradPush* push = nullptr);

// Projection backward of the last forward render with AdamScaled applied to
// the splats in the same kernel (single-GPU trainer step).
bsx_status project_bwd_fused(bsx_ctx* ctx, const float* d_v_combined, float* d_v_transforms, float* d_v_sh,
                             float* d_v_raw_opac, float* d_v_refine, const FusedAdam& adam) {
    const bsx_fwd_state& f = ctx->fwd;
    if (!f.valid) return fail(ctx, BSX_ERR_STATE, "project_bwd needs a preceding render");
    if (3 * f.coeffs > 80) return fail(ctx, BSX_ERR_SHAPE, "fused Adam supports at most 80 SH columns");
    return launch_project_bwd(ctx, f.uni, f.transforms, f.sh, f.raw_opac, f.n, f.coeffs, (int)f.degree, f.mip,
                              d_v_combined, d_v_transforms, d_v_sh, d_v_raw_opac, d_v_refine, &adam);
}

// Projection backward of the last forward render whose gradient rows go
// straight into their owners' exchange slots (data-parallel trainer step).
bsx_status project_bwd_push(bsx_ctx* ctx, const float* d_v_combined, float* d_v_refine, const GradPush& push) {
    const bsx_fwd_state& f = ctx->fwd;
    if (!f.valid) return fail(ctx, BSX_ERR_STATE, "project_bwd needs a preceding render");
    return launch_project_bwd(ctx, f.uni, f.transforms, f.sh, f.raw_opac, f.n, f.coeffs, (int)f.degree, f.mip,
                              d_v_combined, nullptr, nullptr, nullptr, d_v_refine, nullptr, &push);
}

namespace {
int degree_from_coeffs(uint32_t c) {
    for (int d = 0; d <= 4; ++d)
        if ((uint32_t)((d + 1) * (d + 1)) == c) return d;
    return -1;
}
uint32_t bits_for(uint32_t v) { return v == 0 ? 0u : 32u - (uint32_t)__builtin_clz(v); }
}  // namespace

}  // namespace bsx

using namespace bsx;

#define BSX_TRY(expr)                     \
    do {                                  \
        bsx_status _s = (expr);           \
        if (_s != BSX_OK) return _s;      \
    } while (0)

extern "C" {

bsx_status bsx_render_fwd(bsx_ctx* ctx, const bsx_camera* cam, uint32_t w, uint32_t h, const float* d_transforms,
                          const float* d_sh, const float* d_raw_opac, uint32_t n, uint32_t coeffs, int32_t render_mode,
                          int32_t raster_pass, const float background[3], bsx_render_out* out) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    // A render that fails part way leaves no state a backward could consume:
    // the previous render's rows and ranges may already be overwritten.
    ctx->fwd.valid = 0;
    if (!cam || !out || !background) return BSX_ERR_INVALID_ARG;
    if (w == 0 || h == 0) return fail(ctx, BSX_ERR_INVALID_ARG, "Can't render images with 0 size.");
    if (w > 16384 || h > 16384) return fail(ctx, BSX_ERR_CAPACITY, "image side limited to 16384 pixels");
    if (n && (!d_transforms || !d_sh || !d_raw_opac)) return fail(ctx, BSX_ERR_INVALID_ARG, "null splat tensor");
    if (render_mode != BSX_RENDER_DEFAULT && render_mode != BSX_RENDER_MIP)
        return fail(ctx, BSX_ERR_INVALID_ARG, "render_mode");
    if (raster_pass < 0 || raster_pass > 2) return fail(ctx, BSX_ERR_INVALID_ARG, "raster_pass");
    const int degree = degree_from_coeffs(coeffs);
    if (degree < 0) return fail(ctx, BSX_ERR_SHAPE, "sh_coeffs must be [N, (degree+1)^2, 3] with degree <= 4");
    if (((uintptr_t)d_sh | (uintptr_t)d_raw_opac) % 4 || (uintptr_t)d_transforms % 8)
        return fail(ctx, BSX_ERR_INVALID_ARG, "transforms must be 8-byte aligned, sh / opacities 4-byte aligned");
    cudaSetDevice(ctx->device);
    bsx_project_uniforms uni;
    BSX_TRY(bsx_make_project_uniforms(cam, w, h, (uint32_t)degree, n, &uni));
    const int bwd_info = raster_pass != BSX_PASS_FORWARD;
    const int smooth = raster_pass == BSX_PASS_BACKWARD_SMOOTH_CUTOFF;
    const int mip = render_mode == BSX_RENDER_MIP;
    const uint32_t T = uni.tile_bw * uni.tile_bh;
    const size_t P = (size_t)w * h;
    const size_t nn = n ? n : 1;

    BSX_TRY(ensure(ctx, ctx->projected, nn * BSX_PROJECTED_LANES * 4));
    BSX_TRY(ensure(ctx, ctx->counts, nn * 4));
    BSX_TRY(ensure(ctx, ctx->max_radius, nn * 4));
    BSX_TRY(ensure(ctx, ctx->vis_gid, nn * 4));
    BSX_TRY(ensure(ctx, ctx->depth_keys, nn * 4));
    BSX_TRY(ensure(ctx, ctx->depth_order, nn * 4));
    BSX_TRY(ensure(ctx, ctx->cum, nn * 4));
    BSX_TRY(ensure(ctx, ctx->scalars, 64));
    BSX_TRY(ensure(ctx, ctx->tile_offsets, (size_t)T * 2 * 4));
    if (bwd_info) {
        BSX_TRY(ensure(ctx, ctx->image, P * 16));
        BSX_TRY(ensure(ctx, ctx->visible, nn * 4));
    } else {
        BSX_TRY(ensure(ctx, ctx->image_packed, P * 4));
    }
    uint32_t* scalars = ctx->scalars.as<uint32_t>();
    uint32_t V = 0, M = 0;
    if (n) {
        BSX_TRY(launch_project_fwd(ctx, uni, d_transforms, d_sh, d_raw_opac, n, coeffs, degree, mip,
                                   ctx->projected.as<float>(), ctx->counts.as<uint32_t>(), ctx->max_radius.as<float>(),
                                   ctx->vis_gid.as<uint32_t>(), ctx->depth_keys.as<uint32_t>(), scalars,
                                   // scratch: both are rewritten later in the render (depth sort, count scan)
                                   ctx->depth_order.as<uint32_t>(), ctx->cum.as<uint32_t>()));
        // The one host synchronisation of the render (render.rs:308-330).
        BSX_TRY(check_cuda(ctx, cudaMemcpyAsync(ctx->h_pinned, scalars, 8, cudaMemcpyDeviceToHost, ctx->stream),
                           "count readback"));
        BSX_TRY(check_device_error(ctx));
        V = ctx->h_pinned[0];
        M = ctx->h_pinned[1];
    }
    if (V > n) return fail(ctx, BSX_ERR_CAPACITY, "visible count exceeds splat count");
    if ((uint64_t)M > (uint64_t)V * T || M >= (1u << 30))
        return fail(ctx, BSX_ERR_CAPACITY, "intersection count out of range");
    const size_t mm = M ? M : 1;
    BSX_TRY(ensure(ctx, ctx->sort_keys_b, std::max(mm, (size_t)nn) * 4));
    BSX_TRY(ensure(ctx, ctx->sort_vals_b, mm * 4));
    BSX_TRY(ensure(ctx, ctx->isect_tile, mm * 4));
    BSX_TRY(ensure(ctx, ctx->isect_gid, mm * 4));
    if (bwd_info) BSX_TRY(ensure(ctx, ctx->isect_mask, mm));
    uint32_t* depth_order = ctx->depth_order.as<uint32_t>();
    if (V) {
        BSX_TRY(radix_sort_pairs(ctx, ctx->depth_keys.as<uint32_t>(), ctx->vis_gid.as<uint32_t>(), V, 32,
                                 ctx->sort_keys_b.as<uint32_t>(), depth_order));
        BSX_TRY(scan_inclusive_u32(ctx, ctx->counts.as<uint32_t>(), depth_order, V, ctx->cum.as<uint32_t>(), nullptr));
        if (M) {
            BSX_TRY(launch_emit(ctx, ctx->projected.as<float>(), depth_order, ctx->cum.as<uint32_t>(), V, uni.tile_bw,
                                uni.tile_bh, ctx->sort_keys_b.as<uint32_t>(), ctx->sort_vals_b.as<uint32_t>(), M));
            BSX_TRY(radix_sort_pairs(ctx, ctx->sort_keys_b.as<uint32_t>(), ctx->sort_vals_b.as<uint32_t>(), M,
                                     bits_for(T), ctx->isect_tile.as<uint32_t>(), ctx->isect_gid.as<uint32_t>()));
        }
    }
    BSX_TRY(tile_offsets(ctx, ctx->isect_tile.as<uint32_t>(), M, T, ctx->tile_offsets.as<uint32_t>()));
    if (bwd_info)
        BSX_TRY(check_cuda(ctx, cudaMemsetAsync(ctx->visible.p, 0, nn * 4, ctx->stream), "memset visible"));
    BSX_TRY(launch_raster_fwd(ctx, ctx->isect_gid.as<uint32_t>(), ctx->tile_offsets.as<uint32_t>(),
                              ctx->projected.as<float>(), bwd_info ? ctx->image.as<float>() : nullptr,
                              bwd_info ? nullptr : ctx->image_packed.as<uint32_t>(),
                              bwd_info ? ctx->visible.as<float>() : nullptr,
                              bwd_info ? ctx->isect_mask.as<uint8_t>() : nullptr, uni, background, bwd_info, smooth));

    uni.num_visible = V;
    std::memset(out, 0, sizeof *out);
    out->d_image = bwd_info ? ctx->image.as<float>() : nullptr;
    out->d_image_packed = bwd_info ? nullptr : ctx->image_packed.as<uint32_t>();
    out->d_visible = bwd_info ? ctx->visible.as<float>() : nullptr;
    out->d_max_radius = ctx->max_radius.as<float>();
    out->d_tile_offsets = ctx->tile_offsets.as<uint32_t>();
    out->d_projected = ctx->projected.as<float>();
    out->d_isect_gid = ctx->isect_gid.as<uint32_t>();
    out->d_isect_tile = ctx->isect_tile.as<uint32_t>();
    out->d_depth_order = depth_order;
    out->d_tile_counts = ctx->counts.as<uint32_t>();
    out->d_cum_counts = ctx->cum.as<uint32_t>();
    out->num_visible = V;
    out->num_intersections = M;
    out->tile_bw = uni.tile_bw;
    out->tile_bh = uni.tile_bh;
    out->uniforms = uni;

    bsx_fwd_state& f = ctx->fwd;
    f.valid = 1;
    f.bwd_info = bwd_info;
    f.smooth = smooth;
    f.mip = mip;
    f.n = n;
    f.coeffs = coeffs;
    f.degree = (uint32_t)degree;
    f.num_visible = V;
    f.num_intersections = M;
    f.bg[0] = background[0];
    f.bg[1] = background[1];
    f.bg[2] = background[2];
    f.uni = uni;
    f.transforms = d_transforms;
    f.sh = d_sh;
    f.raw_opac = d_raw_opac;
    return BSX_OK;
}

bsx_status bsx_rasterize_bwd(bsx_ctx* ctx, const float* d_v_output, int32_t compute_refine_weight,
                             float* d_v_combined) {
    if (!ctx || !d_v_output || !d_v_combined) return BSX_ERR_INVALID_ARG;
    const bsx_fwd_state& f = ctx->fwd;
    if (!f.valid || !f.bwd_info) return fail(ctx, BSX_ERR_STATE, "rasterize_bwd needs a preceding backward-pass render");
    if (((uintptr_t)d_v_output | (uintptr_t)d_v_combined) % 16)
        return fail(ctx, BSX_ERR_INVALID_ARG, "v_output and v_combined must be 16-byte aligned");
    cudaSetDevice(ctx->device);
    const size_t nn = f.n ? f.n : 1;
    BSX_TRY(check_cuda(ctx, cudaMemsetAsync(d_v_combined, 0, nn * kGradStride * 4, ctx->stream), "memset v_combined"));
    if (f.num_intersections == 0) return BSX_OK;
    return launch_raster_bwd(ctx, ctx->isect_gid.as<uint32_t>(), ctx->tile_offsets.as<uint32_t>(),
                             ctx->projected.as<float>(), ctx->image.as<float>(), d_v_output, d_v_combined,
                             ctx->isect_mask.as<uint8_t>(), ctx->tile_order.as<uint32_t>(), f.uni, f.bg, f.smooth,
                             compute_refine_weight);
}

bsx_status bsx_project_bwd(bsx_ctx* ctx, const float* d_v_combined, float* d_v_transforms, float* d_v_sh,
                           float* d_v_raw_opac, float* d_v_refine) {
    if (!ctx || !d_v_combined || !d_v_transforms || !d_v_sh || !d_v_raw_opac || !d_v_refine) return BSX_ERR_INVALID_ARG;
    const bsx_fwd_state& f = ctx->fwd;
    if (!f.valid) return fail(ctx, BSX_ERR_STATE, "project_bwd needs a preceding render");
    if ((uintptr_t)d_v_combined % 16) return fail(ctx, BSX_ERR_INVALID_ARG, "v_combined must be 16-byte aligned");
    cudaSetDevice(ctx->device);
    return launch_project_bwd(ctx, f.uni, f.transforms, f.sh, f.raw_opac, f.n, f.coeffs, (int)f.degree, f.mip,
                              d_v_combined, d_v_transforms, d_v_sh, d_v_raw_opac, d_v_refine, nullptr);
}

}  // extern "C"
