// ctx.cu - context lifetime, error reporting, workspace growth and the
// host-side camera -> uniforms computation.
#include <cmath>
#include <cstring>
#include <new>

#include "common.cuh"

namespace bsx {

bsx_status fail(bsx_ctx* ctx, bsx_status s, const std::string& msg) {
    if (ctx) ctx->last_error = msg;
    return s;
}

bsx_status check_cuda(bsx_ctx* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return BSX_OK;
    return fail(ctx, BSX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Workspace memory is stream-ordered (cudaMallocAsync / cudaFreeAsync on the
// context's stream, from the device's default pool, which keeps what it
// frees): growing a buffer neither synchronises the device nor waits for the
// stream, and the old buffer is released only after the work queued before it.
void release(bsx_ctx* ctx, DevBuf& b) {
    if (b.p) cudaFreeAsync(b.p, ctx->stream);
    b.p = nullptr;
    b.cap = 0;
}

bsx_status ensure(bsx_ctx* ctx, DevBuf& b, size_t bytes) {
    if (bytes == 0) bytes = 16;
    if (bytes <= b.cap) return BSX_OK;
    size_t nb = bytes + bytes / 2;  // headroom: a growing splat count reallocates rarely
    nb = (nb + 255) & ~size_t(255);
    release(ctx, b);
    cudaError_t e = cudaMallocAsync(&b.p, nb, ctx->stream);
    if (e != cudaSuccess) {
        b.p = nullptr;
        return fail(ctx, BSX_ERR_CUDA, std::string("workspace allocation of ") + std::to_string(nb) +
                                           " bytes failed: " + cudaGetErrorString(e));
    }
    b.cap = nb;
    return BSX_OK;
}

static cudaEvent_t pool_event(bsx_ctx* ctx) {
    if (!ctx->prof_pool.empty()) {
        cudaEvent_t e = ctx->prof_pool.back();
        ctx->prof_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void prof_begin(bsx_ctx* ctx) {
    if (!ctx->profiling) return;
    ctx->prof_start = pool_event(ctx);
    cudaEventRecord(ctx->prof_start, ctx->stream);
}

bsx_status post_launch(bsx_ctx* ctx, const char* name) {
    ctx->launches++;
    if (ctx->profiling && ctx->prof_start) {
        cudaEvent_t end = pool_event(ctx);
        cudaEventRecord(end, ctx->stream);
        ctx->prof_pending.push_back({name, ctx->prof_start, end});
        ctx->prof_start = nullptr;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(ctx, BSX_ERR_CUDA, std::string("launch of ") + name + ": " + cudaGetErrorString(e));
    return BSX_OK;
}

bsx_status check_device_error(bsx_ctx* ctx) {
    cudaError_t e = cudaMemcpyAsync(ctx->h_pinned + 8, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return check_cuda(ctx, e, "error-word readback");
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return check_cuda(ctx, e, "cudaStreamSynchronize");
    int code = (int)ctx->h_pinned[8];
    if (code == 0) return BSX_OK;
    cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream);
    if (code == kDevLookbackTimeout)
        return fail(ctx, BSX_ERR_DEVICE_TIMEOUT, "a bounded device-side lookback wait expired");
    if (code == kDevPeerTimeout)
        return fail(ctx, BSX_ERR_DEVICE_TIMEOUT, "a data-parallel peer did not reach the exchange within the timeout");
    if (code == kDevBadIndex)
        return fail(ctx, BSX_ERR_INVALID_ARG, "an intersection id, tile range or global id was out of bounds (skipped)");
    return fail(ctx, BSX_ERR_CAPACITY, "device-side range check failed (code " + std::to_string(code) + ")");
}

}  // namespace bsx

using namespace bsx;

extern "C" {

int bsx_abi_version(void) { return BSX_ABI_VERSION; }

const char* bsx_status_string(bsx_status s) {
    switch (s) {
        case BSX_OK: return "ok";
        case BSX_ERR_INVALID_ARG: return "invalid argument";
        case BSX_ERR_SHAPE: return "shape mismatch";
        case BSX_ERR_CAPACITY: return "capacity exceeded";
        case BSX_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case BSX_ERR_CUDA: return "CUDA error";
        case BSX_ERR_STATE: return "invalid call order";
        case BSX_ERR_UNSUPPORTED: return "unsupported";
        case BSX_ERR_FORMAT: return "malformed file";
    }
    return "unknown status";
}

bsx_status bsx_create(int device, bsx_ctx** out) {
    if (!out) return BSX_ERR_INVALID_ARG;
    *out = nullptr;
    bsx_ctx* ctx = new (std::nothrow) bsx_ctx();
    if (!ctx) return BSX_ERR_INVALID_ARG;
    ctx->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, 256);
    if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, 256);
    if (e == cudaSuccess) e = cudaMallocHost(&ctx->h_pinned, 64 * sizeof(uint32_t));
    if (e == cudaSuccess) {
        // workspace growth reuses freed blocks instead of returning them to the device
        cudaMemPool_t pool;
        e = cudaDeviceGetDefaultMemPool(&pool, device);
        uint64_t keep = UINT64_MAX;
        if (e == cudaSuccess) e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    if (e != cudaSuccess) {
        if (ctx->d_err) cudaFree(ctx->d_err);
        delete ctx;
        return BSX_ERR_CUDA;
    }
    *out = ctx;
    return BSX_OK;
}

bsx_status bsx_destroy(bsx_ctx* ctx) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    else cudaDeviceSynchronize();
    DevBuf* bufs[] = {&ctx->projected, &ctx->counts, &ctx->depth_keys, &ctx->vis_gid, &ctx->depth_order,
                      &ctx->cum, &ctx->isect_tile, &ctx->isect_gid, &ctx->tile_offsets, &ctx->image,
                      &ctx->image_packed, &ctx->visible, &ctx->max_radius, &ctx->sort_tmp_k, &ctx->sort_tmp_v,
                      &ctx->sort_hist, &ctx->sort_lookback, &ctx->scan_status, &ctx->scalars, &ctx->grad,
                      &ctx->loss_partials, &ctx->loss_planes, &ctx->sort_keys_b, &ctx->sort_vals_b,
                      &ctx->tile_order, &ctx->isect_mask,
                      &ctx->ref_rows,      &ctx->ref_ids,     &ctx->ref_offsets, &ctx->ref_grad, &ctx->ref_order,
                      &ctx->bounds_tmp};
    for (DevBuf* b : bufs) release(ctx, *b);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    else cudaDeviceSynchronize();
    if (ctx->d_err) cudaFree(ctx->d_err);
    if (ctx->h_pinned) cudaFreeHost(ctx->h_pinned);
    for (auto& r : ctx->prof_pending) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (cudaEvent_t e : ctx->prof_pool) cudaEventDestroy(e);
    delete ctx;
    return BSX_OK;
}

bsx_status bsx_trim(bsx_ctx* ctx) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    cudaError_t e = ctx->stream ? cudaStreamSynchronize(ctx->stream) : cudaDeviceSynchronize();
    if (e != cudaSuccess) return check_cuda(ctx, e, "synchronise before trim");
    DevBuf* bufs[] = {&ctx->projected, &ctx->counts, &ctx->depth_keys, &ctx->vis_gid, &ctx->depth_order,
                      &ctx->cum, &ctx->isect_tile, &ctx->isect_gid, &ctx->tile_offsets, &ctx->image,
                      &ctx->image_packed, &ctx->visible, &ctx->max_radius, &ctx->sort_tmp_k, &ctx->sort_tmp_v,
                      &ctx->sort_hist, &ctx->sort_lookback, &ctx->scan_status, &ctx->scalars, &ctx->grad,
                      &ctx->loss_partials, &ctx->loss_planes, &ctx->sort_keys_b, &ctx->sort_vals_b,
                      &ctx->tile_order, &ctx->isect_mask,
                      &ctx->ref_rows,      &ctx->ref_ids,     &ctx->ref_offsets, &ctx->ref_grad, &ctx->ref_order,
                      &ctx->bounds_tmp};
    for (DevBuf* b : bufs) release(ctx, *b);
    ctx->fwd.valid = 0;
    e = ctx->stream ? cudaStreamSynchronize(ctx->stream) : cudaDeviceSynchronize();
    if (e != cudaSuccess) return check_cuda(ctx, e, "synchronise after trim");
    // hand the pool's unused memory back to the device
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, ctx->device) == cudaSuccess) cudaMemPoolTrimTo(pool, 0);
    return BSX_OK;
}

bsx_status bsx_set_stream(bsx_ctx* ctx, void* stream) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    ctx->stream = (cudaStream_t)stream;
    return BSX_OK;
}

bsx_status bsx_sync(bsx_ctx* ctx) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    return check_device_error(ctx);
}

const char* bsx_last_error(const bsx_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

uint64_t bsx_launch_count(const bsx_ctx* ctx) { return ctx ? ctx->launches : 0; }

bsx_status bsx_profile_enable(bsx_ctx* ctx, int32_t on) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    ctx->profiling = on != 0;
    return BSX_OK;
}

bsx_status bsx_profile_collect(bsx_ctx* ctx) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    bsx_status s = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (s != BSX_OK) return s;
    for (auto& r : ctx->prof_pending) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, r.a, r.b);
        size_t i = 0;
        while (i < ctx->prof_names.size() && ctx->prof_names[i] != r.name) ++i;
        if (i == ctx->prof_names.size()) {
            ctx->prof_names.emplace_back(r.name);
            ctx->prof_ms.push_back(0.0);
            ctx->prof_count.push_back(0);
        }
        ctx->prof_ms[i] += ms;
        ctx->prof_count[i] += 1;
        ctx->prof_pool.push_back(r.a);
        ctx->prof_pool.push_back(r.b);
    }
    ctx->prof_pending.clear();
    return BSX_OK;
}

int32_t bsx_profile_count(const bsx_ctx* ctx) { return ctx ? (int32_t)ctx->prof_names.size() : 0; }

bsx_status bsx_profile_entry(const bsx_ctx* ctx, int32_t i, const char** name, double* total_ms, uint64_t* launches) {
    if (!ctx || i < 0 || i >= (int32_t)ctx->prof_names.size()) return BSX_ERR_INVALID_ARG;
    if (name) *name = ctx->prof_names[i].c_str();
    if (total_ms) *total_ms = ctx->prof_ms[i];
    if (launches) *launches = ctx->prof_count[i];
    return BSX_OK;
}

bsx_status bsx_profile_reset(bsx_ctx* ctx) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    bsx_status s = bsx_profile_collect(ctx);
    ctx->prof_names.clear();
    ctx->prof_ms.clear();
    ctx->prof_count.clear();
    return s;
}

// camera.rs:49-101 (focal, centre, world_to_local via glam's Affine3A
// inverse), camera.rs:200-254 (pinhole Jacobian clamp limits) and
// render.rs:116-136 (uniform assembly).
// Per-model focal length and Jacobian clamp (crates/brush-render/src/camera.rs:85-254), in f64 like
// the reference. p holds the model's f32 coefficients (bsx_camera_model).
static double kb4_d(double theta, const float* p) {
    const double t2 = theta * theta, t3 = t2 * theta, t5 = t3 * t2, t7 = t5 * t2, t9 = t7 * t2;
    return theta + (double)p[0] * t3 + (double)p[1] * t5 + (double)p[2] * t7 + (double)p[3] * t9;
}
static double rt8_radial(double r, const float* p) {
    const double r2 = r * r, r4 = r2 * r2, r6 = r4 * r2;
    const double num = 1.0 + (double)p[0] * r2 + (double)p[1] * r4 + (double)p[2] * r6;
    const double den = 1.0 + (double)p[3] * r2 + (double)p[4] * r4 + (double)p[5] * r6;
    return num / den;
}
static double rt8_undistort_radius(double r_d, const float* p) {
    double r = r_d;
    for (int i = 0; i < 30; ++i) {
        const double factor = rt8_radial(r, p);
        if (std::fabs(factor) < 1e-12) break;
        const double r_new = r_d / factor;
        if (std::fabs(r_new - r) < 1e-12) {
            r = r_new;
            break;
        }
        r = r_new;
    }
    return r;
}
static double model_fov_to_focal(double fov, uint32_t pixels, int model, const float* p) {
    const double half = fov / 2.0;
    double proj = std::tan(half);
    if (model == BSX_CAMERA_KANNALA_BRANDT_4 || model == BSX_CAMERA_THIN_PRISM_FISHEYE) proj = kb4_d(half, p);
    else if (model == BSX_CAMERA_RADIAL_TANGENTIAL_8) proj = proj * rt8_radial(proj, p);
    return ((double)pixels / 2.0) / proj;
}
static float rt8_undistort_edge(float edge, const float* p) {
    const float mag = (float)rt8_undistort_radius((double)std::fabs(edge), p);
    return mag * (std::signbit(edge) ? -1.0f : 1.0f);
}

bsx_status bsx_make_project_uniforms(const bsx_camera* cam, uint32_t w, uint32_t h, uint32_t sh_degree,
                                     uint32_t total, bsx_project_uniforms* out) {
    if (!cam || !out || w == 0 || h == 0) return BSX_ERR_INVALID_ARG;
    if (cam->camera_model < BSX_CAMERA_PINHOLE || cam->camera_model > BSX_CAMERA_THIN_PRISM_FISHEYE)
        return BSX_ERR_INVALID_ARG;
    const int model = cam->camera_model;
    const float* kp = cam->model_params;
    // Rotation matrix columns from the (x, y, z, w) quaternion.
    const float qx = cam->rotation[0], qy = cam->rotation[1], qz = cam->rotation[2], qw = cam->rotation[3];
    const float x2 = qx + qx, y2 = qy + qy, z2 = qz + qz;
    const float xx = qx * x2, xy = qx * y2, xz = qx * z2;
    const float yy = qy * y2, yz = qy * z2, zz = qz * z2;
    const float wx = qw * x2, wy = qw * y2, wz = qw * z2;
    const float X[3] = {1.0f - (yy + zz), xy + wz, xz - wy};
    const float Y[3] = {xy - wz, 1.0f - (xx + zz), yz + wx};
    const float Z[3] = {xz + wy, yz - wx, 1.0f - (xx + yy)};
    auto cross = [](const float* a, const float* b, float* o) {
        o[0] = a[1] * b[2] - a[2] * b[1];
        o[1] = a[2] * b[0] - a[0] * b[2];
        o[2] = a[0] * b[1] - a[1] * b[0];
    };
    float t0[3], t1[3], t2[3];
    cross(Y, Z, t0);
    cross(Z, X, t1);
    cross(X, Y, t2);
    const float det = (Z[0] * t2[0] + Z[1] * t2[1]) + Z[2] * t2[2];
    const float inv = 1.0f / det;
    float a[3], b[3], c[3];
    for (int i = 0; i < 3; ++i) {
        a[i] = t0[i] * inv;
        b[i] = t1[i] * inv;
        c[i] = t2[i] * inv;
    }
    // Inverse = transpose of columns (a, b, c): column i is (a[i], b[i], c[i]).
    float cols[3][3];
    for (int i = 0; i < 3; ++i) {
        cols[i][0] = a[i];
        cols[i][1] = b[i];
        cols[i][2] = c[i];
    }
    const float p[3] = {cam->position[0], cam->position[1], cam->position[2]};
    float mp[3];
    for (int k = 0; k < 3; ++k) mp[k] = (cols[0][k] * p[0] + cols[1][k] * p[1]) + cols[2][k] * p[2];
    std::memset(out, 0, sizeof *out);
    for (int i = 0; i < 3; ++i)
        for (int k = 0; k < 3; ++k) out->viewmat[i * 3 + k] = cols[i][k];
    out->viewmat[9] = -mp[0];
    out->viewmat[10] = -mp[1];
    out->viewmat[11] = -mp[2];
    const double fx = model_fov_to_focal(cam->fov_x, w, model, kp);
    const double fy = model_fov_to_focal(cam->fov_y, h, model, kp);
    out->fx = (float)fx;
    out->fy = (float)fy;
    out->cx = cam->center_uv[0] * (float)w;
    out->cy = cam->center_uv[1] * (float)h;
    out->camera_pos[0] = p[0];
    out->camera_pos[1] = p[1];
    out->camera_pos[2] = p[2];
    const float hyp = std::hypot((float)cam->fov_x, (float)cam->fov_y);
    out->half_max_render_fov = fminf(hyp * 1.05f, 2.0f * 3.14159265358979323846f - 1e-6f) * 0.5f;
    const float wf = (float)w, hf = (float)h;
    if (model == BSX_CAMERA_PINHOLE || model == BSX_CAMERA_RADIAL_TANGENTIAL_8) {
        out->lim_pos_x = (1.15f * wf - out->cx) / out->fx;
        out->lim_pos_y = (1.15f * hf - out->cy) / out->fy;
        out->lim_neg_x = (-0.15f * wf - out->cx) / out->fx;
        out->lim_neg_y = (-0.15f * hf - out->cy) / out->fy;
        if (model == BSX_CAMERA_RADIAL_TANGENTIAL_8) {  // undistorted bounds (camera.rs:227-240)
            out->lim_pos_x = rt8_undistort_edge(out->lim_pos_x, kp);
            out->lim_pos_y = rt8_undistort_edge(out->lim_pos_y, kp);
            out->lim_neg_x = rt8_undistort_edge(out->lim_neg_x, kp);
            out->lim_neg_y = rt8_undistort_edge(out->lim_neg_y, kp);
        }
    }  // fisheye models: no clamp, limits stay 0 (camera.rs:241-244)
    out->camera_model = model;
    for (int k = 0; k < BSX_CAMERA_PARAMS; ++k) out->model_params[k] = kp[k];
    out->img_w = w;
    out->img_h = h;
    out->tile_bw = (w + kTile - 1) / kTile;
    out->tile_bh = (h + kTile - 1) / kTile;
    out->sh_degree = sh_degree;
    out->total_splats = total;
    out->num_visible = 0;
    return BSX_OK;
}

}  // extern "C"
