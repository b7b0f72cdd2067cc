// train.cu - the whole training step behind one C entry point.
//
// Restates SplatTrainer::step_with_refine_weight
// (crates/brush-train/src/train.rs:619-1182) for the hot path: backward-pass
// render -> fused SSIM+L1 loss and its gradient (train.rs:729-761) -> raster
// backward -> projection backward -> AdamScaled over transforms / SH /
// opacity with the per-step rate table (train.rs:964-1051) -> RefineRecord
// statistics (stats.rs:111-121). Every stage is a launch of this library on
// the context's stream; the only host synchronisation is the render's count
// readback.
//
// Learning-rate schedules: the reference steps two burn ExponentialLrScheduler
// instances once per optimizer step (train.rs:991-994; burn git main, pinned
// da67c939 in the reference's Cargo.lock). Restated here from burn's published
// definition: the scheduler starts at initial / gamma and each step multiplies
// by gamma (f64) and returns the new rate, so the first step uses the initial
// rate; gamma = (end / start)^(1 / total_train_iters) (train.rs:243-258).
#include <math.h>

#include <algorithm>

#include <vector>

#include "trainer.cuh"

namespace bsx {

bsx_status project_bwd_fused(bsx_ctx* ctx, const float* d_v_combined, float* d_v_transforms, float* d_v_sh,
                             float* d_v_raw_opac, float* d_v_refine, const FusedAdam& adam);
bsx_status project_bwd_push(bsx_ctx* ctx, const float* d_v_combined, float* d_v_refine, const GradPush& push);

namespace {

constexpr int kStatsThreads = 256;

// The mean-noise injection of one step (train.rs:1095-1169), applied after
// AdamScaled: the per-splat arithmetic is bsx_mean_noise (bsx_fmath.h).
struct NoiseArgs {
    float* transforms;      // [N,10], means moved in place
    const float* raw_opac;  // [N], after this step's update
    const float* gate;      // > 0 where the splat may move; null: the visibility statistic just accumulated
    float scale, limit;     // f32(lr_mean) * mean_noise_weight, median bounds size
    uint64_t seed;
    uint32_t step;
};

// raw_op: the splat's opacity logit, loaded by the caller ahead of the gate
__device__ __forceinline__ void noise_row(const NoiseArgs& z, uint32_t i, float gate_src, float raw_op) {
    if (!(gate_src > 0.0f)) return;
    float* m = z.transforms + (size_t)i * 10;
    float mean[3] = {m[0], m[1], m[2]};
    if (bsx_mean_noise(raw_op, 1.0f, z.scale, z.limit, z.seed, z.step, i, mean)) {
        m[0] = mean[0];
        m[1] = mean[1];
        m[2] = mean[2];
    }
}

// RefineRecord::gather_stats (stats.rs:111-121): running MAX of the refine
// weight, SUM of visibility, MAX of the screen-space radius; without a refine
// weight (refine == null) gather_aux_stats (stats.rs:123-127). With NOISE the
// same pass applies the mean noise, gated on the visibility sum it has just
// written (the reference's RefineRecord::vis_mask gate) unless a gate array is
// given.
// View-space gradient statistic of the gradient-threshold densification rule
// (the classic 3DGS densify_and_clone / densify_and_split): the norm of the
// step's screen-space mean gradient in normalised device units, summed over
// the steps in which the splat was visible.
struct Grad2dArgs {
    const float* vgrad;  // raster-backward rows [N,12] (lanes 0-1: d loss / d screen mean, pixels); null: off
    float* accum;        // [N] running sum
    float half_w, half_h;  // d pixel / d ndc
};

template <bool STATS, bool NOISE>
__global__ void __launch_bounds__(kStatsThreads)
    gather_stats_kernel(const float* __restrict__ refine, const float* __restrict__ visible,
                        const float* __restrict__ radius, uint32_t n, float* __restrict__ rmax,
                        float* __restrict__ vsum, float* __restrict__ smax, const NoiseArgs nz, const Grad2dArgs g2) {
    for (uint32_t i = blockIdx.x * kStatsThreads + threadIdx.x; i < n; i += gridDim.x * kStatsThreads) {
        float vs = 0.0f;
        // issued with the statistics' loads rather than after the gate is known
        const float raw_op = NOISE ? __ldg(nz.raw_opac + i) : 0.0f;
        if (STATS) {
            if (refine) rmax[i] = bsx_max(rmax[i], refine[i]);
            const float vi = visible[i];
            vs = vsum[i] + vi;
            vsum[i] = vs;
            smax[i] = bsx_max(smax[i], radius[i]);
            if (g2.vgrad && vi > 0.0f) {
                const float2 v = __ldg(reinterpret_cast<const float2*>(g2.vgrad + (size_t)i * kGradStride));
                const float gx = v.x * g2.half_w, gy = v.y * g2.half_h;
                g2.accum[i] = g2.accum[i] + sqrtf(gx * gx + gy * gy);
            }
        }
        if (NOISE) noise_row(nz, i, nz.gate ? __ldg(nz.gate + i) : vs, raw_op);
    }
}

// Data-parallel steps: this rank's share of the noise gate, before the ranks'
// gates are MAX-combined by the exchange: 1 where the splat was visible in this
// step, or (accum) where the visibility sum including this step is positive.
__global__ void __launch_bounds__(kStatsThreads)
    noise_gate_kernel(const float* __restrict__ visible, const float* __restrict__ vsum, uint32_t n,
                      float* __restrict__ gate) {
    for (uint32_t i = blockIdx.x * kStatsThreads + threadIdx.x; i < n; i += gridDim.x * kStatsThreads) {
        const float v = vsum ? vsum[i] + visible[i] : visible[i];
        gate[i] = v > 0.0f ? 1.0f : 0.0f;
    }
}

__global__ void __launch_bounds__(kStatsThreads) mean_noise_kernel(uint32_t n, const NoiseArgs nz) {
    for (uint32_t i = blockIdx.x * kStatsThreads + threadIdx.x; i < n; i += gridDim.x * kStatsThreads)
        noise_row(nz, i, __ldg(nz.gate + i), __ldg(nz.raw_opac + i));
}

uint32_t stats_blocks(uint32_t n) { return std::min<uint32_t>((n + kStatsThreads - 1) / kStatsThreads, 148 * 8); }

size_t grad_floats(uint32_t n, uint32_t c) { return (size_t)n * (11 + 3 * (size_t)c); }

// Per-step rates: (transform base lr, transform column scales, SH lr, SH
// column scales, opacity lr, lr_mean).
struct Rates {
    float lr_t;
    float t_scale[10];
    float lr_sh;
    std::vector<float> sh_scale;
    float lr_op;
    float lr_mean;
    bool scaled;
};

Rates next_rates(bsx_trainer* tr) {
    Rates r;
    const bsx_train_config& c = tr->cfg;
    if (c.uniform_lr > 0.0f) {
        r.lr_t = r.lr_sh = r.lr_op = r.lr_mean = c.uniform_lr;
        r.scaled = false;
        return r;
    }
    tr->mean_prev *= tr->mean_gamma;
    tr->scale_prev *= tr->scale_gamma;
    const double lr_mean = tr->mean_prev * (double)c.median_scale;
    const double lr_scale = tr->scale_prev;
    r.scaled = true;
    r.lr_t = 1.0f;
    for (int k = 0; k < 3; ++k) r.t_scale[k] = (float)lr_mean;
    for (int k = 3; k < 7; ++k) r.t_scale[k] = (float)c.lr_rotation;
    for (int k = 7; k < 10; ++k) r.t_scale[k] = (float)lr_scale;
    r.lr_sh = (float)c.lr_coeffs_dc;
    r.sh_scale.assign(3 * (size_t)tr->coeffs, 1.0f / c.lr_coeffs_sh_scale);
    for (int k = 0; k < 3; ++k) r.sh_scale[k] = 1.0f;
    r.lr_op = (float)c.lr_opac;
    r.lr_mean = (float)lr_mean;
    return r;
}

// Moments for `rows` rows (zeroed when the layout changes).
bsx_status ensure_moments(bsx_trainer* tr, uint32_t rows, int world, int rank, float** m, float** v) {
    const size_t mv = moment_floats(rows, tr->coeffs);
    if (tr->moment_rows != rows || tr->moment_world != world || tr->moment_rank != rank) {
        bsx_status s = ensure(tr->ctx, tr->moments, mv * 4 + 64);
        if (s != BSX_OK) return s;
        s = check_cuda(tr->ctx, cudaMemsetAsync(tr->moments.p, 0, mv * 4, tr->ctx->stream), "memset moments");
        if (s != BSX_OK) return s;
        tr->moment_rows = rows;
        tr->moment_world = world;
        tr->moment_rank = rank;
        tr->step = 0;
    }
    moment_views(tr->moments.as<float>(), rows, tr->coeffs, m, v);
    return BSX_OK;
}

bsx_loss_cfg loss_cfg_of(const bsx_train_config& c) {
    bsx_loss_cfg l{};
    if (c.ssim_weight > 0.0f) {
        l.l1_weight = 1.0f - c.ssim_weight;
        l.ssim_weight = -c.ssim_weight;
    } else {
        l.l1_weight = 1.0f;
        l.ssim_weight = 0.0f;
    }
    l.composite_bg = 0;
    l.mask = 0;
    return l;
}

// Render -> loss -> raster backward -> projection backward, into the given gradient buffers.
bsx_status forward_backward(bsx_trainer* tr, const bsx_camera* cam, uint32_t w, uint32_t h, const uint32_t* gt,
                            const float* transforms, const float* sh, const float* opac, float* vt, float* vs,
                            float* vo, float* vr, int refine, float* d_loss, bsx_render_out* out,
                            const FusedAdam* adam = nullptr, const GradPush* push = nullptr) {
    bsx_ctx* ctx = tr->ctx;
    bsx_status s = bsx_render_fwd(ctx, cam, w, h, transforms, sh, opac, tr->n, tr->coeffs, tr->cfg.render_mode,
                                  BSX_PASS_BACKWARD, tr->cfg.background, out);
    if (s != BSX_OK) return s;
    s = ensure(ctx, tr->v_output, (size_t)w * h * 16);
    if (s != BSX_OK) return s;
    const bsx_loss_cfg lc = loss_cfg_of(tr->cfg);
    s = bsx_loss_fused(ctx, out->d_image, gt, w, h, &lc, d_loss, tr->v_output.as<float>());
    if (s != BSX_OK) return s;
    s = bsx_rasterize_bwd(ctx, tr->v_output.as<float>(), refine, tr->v_combined.as<float>());
    if (s != BSX_OK) return s;
    if (adam) return project_bwd_fused(ctx, tr->v_combined.as<float>(), vt, vs, vo, vr, *adam);
    if (push) return project_bwd_push(ctx, tr->v_combined.as<float>(), vr, *push);
    return bsx_project_bwd(ctx, tr->v_combined.as<float>(), vt, vs, vo, vr);
}

// Whether this step injects mean noise: configured, and the bounds are valid
// (train.rs:1098: a finite, positive median size).
bool noise_on(const bsx_trainer* tr) {
    const float ms = tr->cfg.median_scale;
    return tr->cfg.mean_noise && bsx_is_finite(ms) && ms > 0.0f && tr->n > 0;
}

NoiseArgs noise_args(const bsx_trainer* tr, float* transforms, const float* raw_opac, const float* gate,
                     float lr_mean) {
    NoiseArgs z;
    z.transforms = transforms;
    z.raw_opac = raw_opac;
    z.gate = gate;
    z.scale = lr_mean * tr->cfg.mean_noise_weight;
    z.limit = tr->cfg.median_scale;
    z.seed = tr->cfg.noise_seed;
    z.step = tr->step;
    return z;
}

// The step's epilogue: RefineRecord statistics and the mean noise in one pass.
// gate: the noise gate array (null: the statistic's visibility sum when the
// accumulated gate is configured, else this step's visible[]).
bsx_status step_epilogue(bsx_trainer* tr, const float* refine, const bsx_render_out& out, float* transforms,
                         const float* raw_opac, const float* gate, float lr_mean) {
    const bool stats = tr->cfg.gather_stats != 0, noise = noise_on(tr);
    if ((!stats && !noise) || tr->n == 0) return BSX_OK;
    if (noise && !gate && !(stats && tr->cfg.noise_vis_gate)) gate = out.d_visible;
    const NoiseArgs nz = noise ? noise_args(tr, transforms, raw_opac, gate, lr_mean) : NoiseArgs{};
    float* st = stats ? tr->stats.as<float>() : nullptr;
    const size_t n = tr->n;
    float* rmax = st;
    float* vsum = st ? st + n : nullptr;
    float* smax = st ? st + 2 * n : nullptr;
    Grad2dArgs g2{nullptr, nullptr, 0.0f, 0.0f};
    if (stats && tr->cfg.accumulate_grad2d) {
        g2.vgrad = tr->v_combined.as<float>();
        g2.accum = st + 3 * n;
        g2.half_w = 0.5f * (float)out.uniforms.img_w;
        g2.half_h = 0.5f * (float)out.uniforms.img_h;
    }
    const uint32_t blocks = stats_blocks(tr->n);
    cudaStream_t s = tr->ctx->stream;
    prof_begin(tr->ctx);
    if (stats && noise)
        gather_stats_kernel<true, true><<<blocks, kStatsThreads, 0, s>>>(refine, out.d_visible, out.d_max_radius,
                                                                         tr->n, rmax, vsum, smax, nz, g2);
    else if (stats)
        gather_stats_kernel<true, false><<<blocks, kStatsThreads, 0, s>>>(refine, out.d_visible, out.d_max_radius,
                                                                          tr->n, rmax, vsum, smax, nz, g2);
    else
        gather_stats_kernel<false, true><<<blocks, kStatsThreads, 0, s>>>(refine, out.d_visible, out.d_max_radius,
                                                                          tr->n, rmax, vsum, smax, nz, g2);
    return post_launch(tr->ctx, "gather_stats_kernel");
}

bsx_status check_cfg(const bsx_train_config* c) {
    if (!c) return BSX_ERR_INVALID_ARG;
    if (c->uniform_lr > 0.0f) return BSX_OK;
    if (!(c->lr_mean > 0.0) || !(c->lr_mean_end > 0.0) || !(c->lr_coeffs_sh_scale > 0.0f) ||
        c->total_train_iters == 0)
        return BSX_ERR_INVALID_ARG;
    return BSX_OK;
}

}  // namespace

}  // namespace bsx

using namespace bsx;

extern "C" {

bsx_status bsx_trainer_create(bsx_ctx* ctx, uint32_t n, uint32_t coeffs, const bsx_train_config* cfg,
                              bsx_trainer** out) {
    if (!ctx || !out || coeffs == 0) return BSX_ERR_INVALID_ARG;
    *out = nullptr;
    if (check_cfg(cfg) != BSX_OK) return fail(ctx, BSX_ERR_INVALID_ARG, "invalid train config");
    bsx_trainer* tr = new (std::nothrow) bsx_trainer();
    if (!tr) return BSX_ERR_CAPACITY;
    tr->ctx = ctx;
    tr->n = n;
    tr->coeffs = coeffs;
    tr->cfg = *cfg;
    if (cfg->uniform_lr <= 0.0f) {
        const double t = (double)cfg->total_train_iters;
        tr->mean_gamma = pow(cfg->lr_mean_end / cfg->lr_mean, 1.0 / t);
        tr->scale_gamma =
            (cfg->lr_scale > 0.0 && cfg->lr_scale_end > 0.0) ? pow(cfg->lr_scale_end / cfg->lr_scale, 1.0 / t) : 1.0;
        tr->mean_prev = cfg->lr_mean / tr->mean_gamma;
        tr->scale_prev = cfg->lr_scale / tr->scale_gamma;
    }
    cudaSetDevice(ctx->device);
    const size_t nn = n ? n : 1;
    bsx_status s = ensure(ctx, tr->v_combined, nn * BSX_GRAD_STRIDE * 4);
    if (s == BSX_OK && cfg->gather_stats) {
        s = ensure(ctx, tr->stats, kRecordArrays * nn * 4);
        if (s == BSX_OK)
            s = check_cuda(ctx, cudaMemsetAsync(tr->stats.p, 0, kRecordArrays * nn * 4, ctx->stream),
                           "memset refine record");
    }
    if (s != BSX_OK) {
        bsx_trainer_destroy(tr);
        return s;
    }
    *out = tr;
    return BSX_OK;
}

bsx_status bsx_trainer_destroy(bsx_trainer* tr) {
    if (!tr) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(tr->ctx->device);
    if (tr->ctx->stream) cudaStreamSynchronize(tr->ctx->stream);
    DevBuf* bufs[] = {&tr->grads, &tr->v_combined, &tr->v_output, &tr->stats, &tr->moments, &tr->moments_next,
                      &tr->plan_keep, &tr->plan_split, &tr->plan_scratch};
    for (DevBuf* b : bufs) release(tr->ctx, *b);
    if (tr->ctx->stream) cudaStreamSynchronize(tr->ctx->stream);
    delete tr;
    return BSX_OK;
}

bsx_status bsx_trainer_optimizer_state(bsx_trainer* tr, float** mt, float** ms, float** mo, float** vt, float** vs,
                                       float** vo, uint32_t* rows) {
    if (!tr || !mt || !ms || !mo || !vt || !vs || !vo || !rows) return BSX_ERR_INVALID_ARG;
    float* m[3] = {nullptr, nullptr, nullptr};
    float* v[3] = {nullptr, nullptr, nullptr};
    if (tr->moment_rows && tr->moments.p) moment_views(tr->moments.as<float>(), tr->moment_rows, tr->coeffs, m, v);
    *mt = m[0];
    *ms = m[1];
    *mo = m[2];
    *vt = v[0];
    *vs = v[1];
    *vo = v[2];
    *rows = tr->moment_rows;
    return BSX_OK;
}

bsx_status bsx_trainer_load_optimizer_state(bsx_trainer* tr, const float* mt, const float* ms, const float* mo,
                                            const float* vt, const float* vs, const float* vo, uint32_t rows,
                                            int32_t world, int32_t rank) {
    if (!tr || world < 1 || world > BSX_MAX_RANKS || rank < 0 || rank >= world) return BSX_ERR_INVALID_ARG;
    if (rows && (!mt || !ms || !mo || !vt || !vs || !vo)) return BSX_ERR_INVALID_ARG;
    bsx_ctx* ctx = tr->ctx;
    const uint32_t rb = (uint32_t)((uint64_t)tr->n * rank / world), re = (uint32_t)((uint64_t)tr->n * (rank + 1) / world);
    if (rows != re - rb) return fail(ctx, BSX_ERR_SHAPE, "optimizer state rows do not match the shard of this rank");
    cudaSetDevice(ctx->device);
    bsx_status s = ensure(ctx, tr->moments, moment_floats(rows, tr->coeffs) * 4 + 64);
    if (s != BSX_OK) return s;
    float* m[3];
    float* v[3];
    moment_views(tr->moments.as<float>(), rows, tr->coeffs, m, v);
    const float* src[6] = {mt, ms, mo, vt, vs, vo};
    float* dst[6] = {m[0], m[1], m[2], v[0], v[1], v[2]};
    const size_t cols[6] = {10, 3 * (size_t)tr->coeffs, 1, 10, 1, 1};
    for (int k = 0; k < 6 && rows; ++k) {
        s = check_cuda(ctx, cudaMemcpyAsync(dst[k], src[k], (size_t)rows * cols[k] * 4, cudaMemcpyDeviceToDevice,
                                            ctx->stream),
                       "load optimizer state");
        if (s != BSX_OK) return s;
    }
    tr->moment_rows = rows;
    tr->moment_world = world;
    tr->moment_rank = rank;
    return BSX_OK;
}

bsx_status bsx_trainer_reserve(bsx_trainer* tr, uint32_t max_splats) {
    if (!tr) return BSX_ERR_INVALID_ARG;
    bsx_ctx* ctx = tr->ctx;
    cudaSetDevice(ctx->device);
    const size_t m = std::max<uint32_t>(max_splats, 1), c3 = 3 * (size_t)tr->coeffs;
    // Sizes each ensure() caller asks for at m splats (render, raster backward,
    // trainer, refine), so none of them reallocates below max_splats.
    struct R {
        DevBuf* b;
        size_t bytes;
    } rs[] = {{&ctx->projected, m * BSX_PROJECTED_LANES * 4},
              {&ctx->counts, m * 4},
              {&ctx->max_radius, m * 4},
              {&ctx->vis_gid, m * 4},
              {&ctx->depth_keys, m * 4},
              {&ctx->depth_order, m * 4},
              {&ctx->cum, m * 4},
              {&ctx->visible, m * 4},
              {&tr->grads, (m * (11 + c3) + m) * 4 + 64},
              {&tr->v_combined, m * BSX_GRAD_STRIDE * 4},
              {&tr->stats, kRecordArrays * m * 4},
              {&tr->moments, moment_floats((uint32_t)m, tr->coeffs) * 4 + 64},
              {&tr->moments_next, moment_floats((uint32_t)m, tr->coeffs) * 4 + 64},
              {&tr->plan_keep, (m + 1) * 4},
              {&tr->plan_split, (m + 1) * 4},
              {&tr->plan_scratch, (m * 6 + 32) * 4}};
    for (const R& r : rs) {
        if (r.bytes <= r.b->cap) continue;
        // keep the contents of live buffers (moments, statistics) across the growth
        DevBuf grown;
        bsx_status s = ensure(ctx, grown, r.bytes);
        if (s != BSX_OK) return s;
        if (r.b->p)
            s = check_cuda(ctx, cudaMemcpyAsync(grown.p, r.b->p, r.b->cap, cudaMemcpyDeviceToDevice, ctx->stream),
                           "copy on reserve");
        if (s != BSX_OK) return s;
        release(ctx, *r.b);
        *r.b = grown;
    }
    return BSX_OK;
}

bsx_status bsx_trainer_set_median_scale(bsx_trainer* tr, float median_scale) {
    if (!tr || !(median_scale > 0.0f)) return BSX_ERR_INVALID_ARG;
    tr->cfg.median_scale = median_scale;
    return BSX_OK;
}

bsx_status bsx_trainer_grad2d_accum(bsx_trainer* tr, float** d_accum) {
    if (!tr || !d_accum) return BSX_ERR_INVALID_ARG;
    if (!tr->cfg.gather_stats) return fail(tr->ctx, BSX_ERR_STATE, "trainer created without gather_stats");
    *d_accum = tr->stats.as<float>() + 3 * (size_t)tr->n;
    return BSX_OK;
}

bsx_status bsx_trainer_stats_buffers(bsx_trainer* tr, float** rmax, float** vsum, float** smax) {
    if (!tr || !rmax || !vsum || !smax) return BSX_ERR_INVALID_ARG;
    if (!tr->cfg.gather_stats) return fail(tr->ctx, BSX_ERR_STATE, "trainer created without gather_stats");
    float* st = tr->stats.as<float>();
    *rmax = st;
    *vsum = st + tr->n;
    *smax = st + 2 * (size_t)tr->n;
    return BSX_OK;
}

bsx_status bsx_trainer_grad_buffers(bsx_trainer* tr, float** vt, float** vs, float** vo, float** vr) {
    if (!tr || !vt || !vs || !vo || !vr) return BSX_ERR_INVALID_ARG;
    // allocated on first use: the data-parallel step writes into the exchange buffers instead
    bsx_status s = ensure(tr->ctx, tr->grads, (grad_floats(tr->n, tr->coeffs) + tr->n) * 4 + 64);
    if (s != BSX_OK) return s;
    float* g = tr->grads.as<float>();
    *vt = g;
    *vs = g + (size_t)tr->n * 10;
    *vo = *vs + (size_t)tr->n * 3 * tr->coeffs;
    *vr = *vo + tr->n;
    return BSX_OK;
}

bsx_status bsx_trainer_raster_grads(bsx_trainer* tr, float** d_v_combined) {
    if (!tr || !d_v_combined) return BSX_ERR_INVALID_ARG;
    *d_v_combined = tr->v_combined.as<float>();
    return BSX_OK;
}

bsx_status bsx_trainer_keep_gradients(bsx_trainer* tr, int32_t on) {
    if (!tr) return BSX_ERR_INVALID_ARG;
    tr->keep_grads = on ? 1 : 0;
    return BSX_OK;
}

bsx_status bsx_train_step(bsx_trainer* tr, const bsx_camera* cam, uint32_t w, uint32_t h, const uint32_t* gt,
                          float* transforms, float* sh, float* opac, int32_t refine, float* d_loss,
                          bsx_train_stats* stats) {
    if (!tr || !cam || !gt || !d_loss || (tr->n && (!transforms || !sh || !opac))) return BSX_ERR_INVALID_ARG;
    bsx_ctx* ctx = tr->ctx;
    tr->planned = false;
    cudaSetDevice(ctx->device);
    float *vt, *vs, *vo, *vr;
    bsx_status s0 = bsx_trainer_grad_buffers(tr, &vt, &vs, &vo, &vr);
    if (s0 != BSX_OK) return s0;
    // The moments and this step's rates are settled before the backward, which
    // applies AdamScaled to every splat row as soon as its gradient exists
    // (no dense gradient round trip through memory; bsx_adam_step arithmetic).
    float* m[3];
    float* v[3];
    bsx_status s = ensure_moments(tr, tr->n, 1, 0, m, v);
    if (s != BSX_OK) return s;
    const Rates r = next_rates(tr);
    tr->step++;
    FusedAdam fa;
    fa.m_t = m[0];
    fa.m_sh = m[1];
    fa.m_o = m[2];
    fa.v_t = v[0];
    fa.v_sh = v[1];
    fa.v_o = v[2];
    fa.lr_t = r.lr_t;
    fa.lr_sh = r.lr_sh;
    fa.lr_op = r.lr_op;
    fa.has_t_scale = r.scaled;
    fa.has_sh_scale = r.scaled;
    for (int k = 0; k < 10; ++k) fa.t_scale[k] = r.scaled ? r.t_scale[k] : 1.0f;
    for (int k = 0; k < 80; ++k) fa.sh_scale[k] = (r.scaled && k < (int)r.sh_scale.size()) ? r.sh_scale[k] : 1.0f;
    fa.b1 = 0.9f;
    fa.b2 = 0.999f;
    fa.eps = 1e-15f;
    fa.inv_bc1 = adam_inv_bias_correction(0.9f, tr->step);
    fa.inv_bc2 = adam_inv_bias_correction(0.999f, tr->step);
    fa.gscale = 1.0f;
    fa.first = tr->step == 1;
    fa.keep_grads = tr->keep_grads;
    bsx_render_out out{};
    s = forward_backward(tr, cam, w, h, gt, transforms, sh, opac, vt, vs, vo, vr, refine, d_loss, &out, &fa);
    if (s != BSX_OK) return s;
    s = step_epilogue(tr, refine ? vr : nullptr, out, transforms, opac, nullptr, r.lr_mean);
    if (s != BSX_OK) return s;
    if (stats) {
        stats->num_visible = out.num_visible;
        stats->num_intersections = out.num_intersections;
        stats->lr_mean = r.lr_mean;
        stats->step = tr->step;
    }
    return BSX_OK;
}

bsx_status bsx_train_step_dp(bsx_trainer* tr, const bsx_camera* cam, uint32_t w, uint32_t h, const uint32_t* gt,
                             const bsx_dp_exchange* ex, const bsx_dp_splats* sp, int32_t refine, float* d_loss,
                             bsx_train_stats* stats) {
    if (!tr || !cam || !gt || !ex || !sp || !d_loss) return BSX_ERR_INVALID_ARG;
    bsx_ctx* ctx = tr->ctx;
    tr->planned = false;
    const int rank = ex->rank, world = ex->world;
    if (world < 1 || world > BSX_MAX_RANKS || rank < 0 || rank >= world)
        return fail(ctx, BSX_ERR_INVALID_ARG, "rank / world out of range (world <= 8)");
    if (!ex->d_refine[rank]) return fail(ctx, BSX_ERR_INVALID_ARG, "the exchange needs refine-weight buffers");
    cudaSetDevice(ctx->device);
    // Gradient push into the owners' slots: needs slots for every shard row,
    // 16-byte aligned slot starts, and shards of at least one projection block
    // (128 rows) so that a block's rows span at most two owners.
    const uint32_t slot = ex->grad_slot_rows;
    // multicast form: every rank writes its dense gradient; the exchange reduces in the switch
    const bool mc = sp->mc_transforms && sp->mc_sh_coeffs && sp->mc_raw_opac && sp->mc_v_transforms &&
                    sp->mc_v_sh_coeffs && sp->mc_v_raw_opac;
    bool push = !mc && world > 1 && slot > 0 && !tr->keep_grads;
    for (int q = 0; push && q < world; ++q) {
        const uint32_t rows = shard_begin(tr->n, q + 1, world) - shard_begin(tr->n, q, world);
        push = rows >= 128 && rows <= slot && slot % 4 == 0 && sp->d_v_transforms[q] && sp->d_v_sh_coeffs[q] &&
               sp->d_v_raw_opac[q];
    }
    GradPush gp{};
    if (push) {
        for (int q = 0; q < world; ++q) {
            gp.dst[0][q] = sp->d_v_transforms[q];
            gp.dst[1][q] = sp->d_v_sh_coeffs[q];
            gp.dst[2][q] = sp->d_v_raw_opac[q];
        }
        gp.n = tr->n;
        gp.slot_rows = slot;
        gp.world = world;
        gp.rank = rank;
    }
    bsx_render_out out{};
    bsx_status s = forward_backward(tr, cam, w, h, gt, sp->d_transforms[rank], sp->d_sh_coeffs[rank],
                                    sp->d_raw_opac[rank], sp->d_v_transforms[rank], sp->d_v_sh_coeffs[rank],
                                    sp->d_v_raw_opac[rank], ex->d_refine[rank], refine, d_loss, &out, nullptr,
                                    push ? &gp : nullptr);
    if (s != BSX_OK) return s;
    const uint32_t rb = (uint32_t)((uint64_t)tr->n * rank / world), re = (uint32_t)((uint64_t)tr->n * (rank + 1) / world);
    float* m[3];
    float* v[3];
    s = ensure_moments(tr, re - rb, world, rank, m, v);
    if (s != BSX_OK) return s;
    const Rates r = next_rates(tr);
    tr->step++;
    bsx_dp_group g[3];
    const float* lrs[3] = {&r.lr_t, &r.lr_sh, &r.lr_op};
    const float* scales[3] = {r.scaled ? r.t_scale : nullptr, r.scaled ? r.sh_scale.data() : nullptr, nullptr};
    const uint32_t cols[3] = {10, 3 * tr->coeffs, 1};
    for (int i = 0; i < 3; ++i) {
        for (int q = 0; q < BSX_MAX_RANKS; ++q) {
            const bool in = q < world;
            g[i].d_param[q] = !in ? nullptr : i == 0 ? sp->d_transforms[q] : i == 1 ? sp->d_sh_coeffs[q] : sp->d_raw_opac[q];
            g[i].d_grad[q] = !in ? nullptr : i == 0 ? sp->d_v_transforms[q] : i == 1 ? sp->d_v_sh_coeffs[q] : sp->d_v_raw_opac[q];
        }
        g[i].d_param_mc = !mc ? nullptr : i == 0 ? sp->mc_transforms : i == 1 ? sp->mc_sh_coeffs : sp->mc_raw_opac;
        g[i].d_grad_mc = !mc ? nullptr : i == 0 ? sp->mc_v_transforms : i == 1 ? sp->mc_v_sh_coeffs : sp->mc_v_raw_opac;
        g[i].d_m = m[i];
        g[i].d_v = v[i];
        g[i].rows = tr->n;
        g[i].cols = cols[i];
        g[i].lr = *lrs[i];
        g[i].h_col_scale = scales[i];
        g[i].reduce_moment_2 = i == 1;
    }
    bsx_dp_exchange e = *ex;
    e.refine_rows = refine ? tr->n : 0;
    e.epoch = ++tr->dp_epoch;
    e.grad_slot_rows = push ? slot : 0;
    if (!mc) e.d_refine_mc = e.d_gate_mc = nullptr;
    // The noise moves a splat where any rank's gate is set, so that every
    // replica applies the same update: this rank's gate goes into its exchange
    // row and the exchange combines the ranks' gates by MAX.
    const bool noise = noise_on(tr);
    e.gate_rows = 0;
    if (noise) {
        if (!ex->d_gate[rank]) return fail(ctx, BSX_ERR_INVALID_ARG, "the mean noise needs gate buffers");
        const float* vsum = (tr->cfg.gather_stats && tr->cfg.noise_vis_gate) ? tr->stats.as<float>() + tr->n : nullptr;
        prof_begin(ctx);
        noise_gate_kernel<<<stats_blocks(tr->n), kStatsThreads, 0, ctx->stream>>>(out.d_visible, vsum, tr->n,
                                                                                 ex->d_gate[rank]);
        s = post_launch(ctx, "noise_gate_kernel");
        if (s != BSX_OK) return s;
        e.gate_rows = tr->n;
    }
    const bsx_adam_cfg ac{0.9f, 0.999f, 1e-15f, tr->step, 1.0f / (float)world};
    s = bsx_dp_adam_step(ctx, &e, g, 3, &ac);
    if (s != BSX_OK) return s;
    s = step_epilogue(tr, refine ? ex->d_refine[rank] : nullptr, out, sp->d_transforms[rank], sp->d_raw_opac[rank],
                      noise ? ex->d_gate[rank] : nullptr, r.lr_mean);
    if (s != BSX_OK) return s;
    if (stats) {
        stats->num_visible = out.num_visible;
        stats->num_intersections = out.num_intersections;
        stats->lr_mean = r.lr_mean;
        stats->step = tr->step;
    }
    return BSX_OK;
}

bsx_status bsx_mean_noise_step(bsx_ctx* ctx, float* d_transforms, const float* d_raw_opac, const float* d_gate,
                               uint32_t n, float scale, float limit, uint64_t seed, uint32_t step) {
    if (!ctx) return BSX_ERR_INVALID_ARG;
    if (n == 0) return BSX_OK;
    if (!d_transforms || !d_raw_opac || !d_gate) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    NoiseArgs z;
    z.transforms = d_transforms;
    z.raw_opac = d_raw_opac;
    z.gate = d_gate;
    z.scale = scale;
    z.limit = limit;
    z.seed = seed;
    z.step = step;
    prof_begin(ctx);
    mean_noise_kernel<<<stats_blocks(n), kStatsThreads, 0, ctx->stream>>>(n, z);
    return post_launch(ctx, "mean_noise_kernel");
}

}  // extern "C"
