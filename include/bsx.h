/*
 * bsx.h - C ABI of the B200 splat-training hot path.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, never
 * throws or unwinds, and returns a bsx_status. Pointers named d_* are CUDA
 * device pointers owned by the caller; h_* are host pointers. All GPU work
 * is enqueued asynchronously on the context's stream (bsx_set_stream); the
 * only host synchronisation inside the library is the one read of the
 * visible/intersection counts per forward render (the reference performs
 * the same read, crates/brush-render/src/render.rs:308-330).
 *
 * Layouts are the reference's (crates/brush-render/src/gaussian_splats.rs:110-127):
 *   transforms [N,10] = mean xyz, quaternion (w,x,y,z) unnormalised, log-scale xyz
 *   sh_coeffs  [N,C,3] coefficient-major, RGB-minor, C = (degree+1)^2
 *   raw_opac   [N]     opacity logits
 *   image      [H,W,4] RGBA float (backward passes) or [H,W] packed RGBA8 (forward pass)
 *   gt         [H,W]   packed RGBA8, r in the low byte
 */
#ifndef BSX_H
#define BSX_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BSX_API __attribute__((visibility("default")))
#else
#define BSX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define BSX_ABI_VERSION 7
/* Gradient lanes per splat written by the raster backward:
 * xy(2) conic(3) rgb(3) alpha refine depth. Reference:
 * crates/brush-render-bwd/src/kernels/rasterize_backwards.rs:40 */
#define BSX_COMPACT_GRAD_LANES 11
/* Row stride of the gradient buffer exchanged between bsx_rasterize_bwd and
 * bsx_project_bwd: the 11 reference lanes plus one pad lane, so each row is
 * three 16-byte words (the raster backward accumulates with vector atomics). */
#define BSX_GRAD_STRIDE 12
/* Row stride (floats) of the projected-splat buffer: xy, conic(3), opacity,
 * rgb, depth, then two pad lanes so each row is three aligned 16-byte words.
 * The reference packs the same first ten lanes (kernels/helpers.rs:48-52). */
#define BSX_PROJECTED_LANES 12
#define BSX_TILE_WIDTH 16

typedef enum bsx_status {
    BSX_OK = 0,
    BSX_ERR_INVALID_ARG = 1,   /* null pointer, bad enum, size out of range */
    BSX_ERR_SHAPE = 2,         /* inconsistent tensor sizes (reference DimCheck) */
    BSX_ERR_CAPACITY = 3,      /* an internal size limit was exceeded */
    BSX_ERR_DEVICE_TIMEOUT = 4,/* a bounded device-side wait gave up */
    BSX_ERR_CUDA = 5,          /* a CUDA runtime call failed */
    BSX_ERR_STATE = 6,         /* call order violated (e.g. backward without forward) */
    BSX_ERR_UNSUPPORTED = 7,   /* valid request this build does not implement */
    BSX_ERR_FORMAT = 8         /* malformed or unsupported file contents (PLY import) */
} bsx_status;

typedef enum bsx_render_mode { BSX_RENDER_DEFAULT = 0, BSX_RENDER_MIP = 1 } bsx_render_mode;

/* crates/brush-render/src/gaussian_splats.rs:46-66 */
typedef enum bsx_raster_pass {
    BSX_PASS_FORWARD = 0,               /* packed RGBA8 output, no bookkeeping */
    BSX_PASS_BACKWARD = 1,              /* RGBA f32 + visible + shortened tile ranges */
    BSX_PASS_BACKWARD_SMOOTH_CUTOFF = 2 /* as BACKWARD with the C^1 alpha-cutoff ramp */
} bsx_raster_pass;

/* crates/brush-render/src/kernels/camera_model/mod.rs:30-37; the distortion
 * coefficients travel in model_params (unused entries ignored):
 *   KANNALA_BRANDT_4   k1 k2 k3 k4                    (kannala_brandt_4.rs:11-16)
 *   RADIAL_TANGENTIAL_8 k1 k2 k3 k4 k5 k6 p1 p2       (radial_tangential_8.rs:11-20)
 *   THIN_PRISM_FISHEYE k1 k2 k3 k4 p1 p2 sx1 sy1      (thin_prism_fisheye.rs:22-29) */
typedef enum bsx_camera_model {
    BSX_CAMERA_PINHOLE = 0,
    BSX_CAMERA_KANNALA_BRANDT_4 = 1,
    BSX_CAMERA_RADIAL_TANGENTIAL_8 = 2,
    BSX_CAMERA_THIN_PRISM_FISHEYE = 3
} bsx_camera_model;
#define BSX_CAMERA_PARAMS 8

/* crates/brush-render/src/camera.rs:11-19 */
typedef struct bsx_camera {
    double fov_x;          /* radians */
    double fov_y;
    float center_uv[2];    /* principal point as a fraction of the image size */
    float position[3];     /* camera centre, world space */
    float rotation[4];     /* camera-to-world rotation quaternion (x, y, z, w) */
    int32_t camera_model;  /* bsx_camera_model */
    float model_params[BSX_CAMERA_PARAMS];
} bsx_camera;

/* crates/brush-render/src/kernels/types.rs:53-83 (ProjectUniforms). */
typedef struct bsx_project_uniforms {
    float viewmat[12];     /* world-to-camera 3x4, column-major: 3 rotation columns + translation */
    float fx, fy, cx, cy;  /* pinhole intrinsics in pixels */
    float camera_pos[3];
    float half_max_render_fov;
    float lim_pos_x, lim_pos_y, lim_neg_x, lim_neg_y; /* projection-Jacobian clamp */
    uint32_t img_w, img_h;
    uint32_t tile_bw, tile_bh;
    uint32_t sh_degree;
    uint32_t total_splats;
    uint32_t num_visible;
    int32_t camera_model;  /* bsx_camera_model */
    float model_params[BSX_CAMERA_PARAMS];
} bsx_project_uniforms;

/* Device outputs of one forward render (crates/brush-render/src/render_aux.rs:16-68).
 * All pointers reference context-owned memory valid until the next render on
 * the same context. Projected rows, visibility, radii and gradients are
 * indexed by the global splat id, so global_from_compact_gid is the identity
 * and compact_gid_from_isect holds global ids. */
typedef struct bsx_render_out {
    float* d_image;                 /* [H,W,4] f32 (backward passes) */
    uint32_t* d_image_packed;       /* [H,W] RGBA8 (forward pass) */
    float* d_visible;               /* [N] 1.0 where a splat was composited (backward passes) */
    float* d_max_radius;            /* [N] max(ex/W, ey/H) for visible splats, else 0 */
    uint32_t* d_tile_offsets;       /* [ty,tx,2] start/end per tile (end shortened in backward passes) */
    float* d_projected;             /* [N, BSX_PROJECTED_LANES] */
    uint32_t* d_isect_gid;          /* [num_intersections] splat id per intersection, tile-major, front-to-back */
    uint32_t* d_isect_tile;         /* [num_intersections] sorted tile id per intersection */
    uint32_t* d_depth_order;        /* [num_visible] visible splat ids sorted by depth */
    uint32_t* d_tile_counts;        /* [N] contributing-tile count per splat */
    uint32_t* d_cum_counts;         /* [num_visible] inclusive scan of counts in depth order */
    uint32_t num_visible;
    uint32_t num_intersections;
    uint32_t tile_bw, tile_bh;
    bsx_project_uniforms uniforms;
} bsx_render_out;

/* crates/brush-loss/src/lib.rs:935-941 (ImageLossConfig). */
typedef struct bsx_loss_cfg {
    float l1_weight;
    float ssim_weight;
    int32_t composite_bg;  /* 1: gt_eff = gt + (1 - gt.a) * bg */
    float bg[3];
    int32_t mask;          /* 1: multiply the loss map by gt.a */
} bsx_loss_cfg;

/* One parameter tensor for the fused Adam update
 * (crates/brush-train/src/adam_scaled.rs:216-383). Rows x cols elements,
 * row-major. col_scale (cols entries, host) multiplies the learning rate per
 * column; reduce_moment_2 keeps one second moment per row (mean of g^2 over
 * the row) as the reference does for the SH coefficients. */
typedef struct bsx_adam_group {
    float* d_param;
    const float* d_grad;
    float* d_m;            /* [rows, cols] */
    float* d_v;            /* [rows, cols] or [rows] when reduce_moment_2 */
    uint32_t rows, cols;
    float lr;
    const float* h_col_scale;  /* may be NULL (all ones); at most 80 entries */
    int32_t reduce_moment_2;
} bsx_adam_group;

typedef struct bsx_adam_cfg {
    float beta_1;          /* 0.9 */
    float beta_2;          /* 0.999 */
    float epsilon;         /* 1e-15 in the reference trainer */
    uint32_t step;         /* time step AFTER this update (1 for the first update) */
    float grad_scale;      /* multiplies every gradient first (1/world_size after a sum all-reduce) */
} bsx_adam_cfg;

/* ---- context ----------------------------------------------------------- */
typedef struct bsx_ctx bsx_ctx;

BSX_API bsx_status bsx_create(int device, bsx_ctx** out);
BSX_API bsx_status bsx_destroy(bsx_ctx* ctx);
BSX_API bsx_status bsx_set_stream(bsx_ctx* ctx, void* cuda_stream);
/* Free the context's grow-only workspace (synchronises its stream); it is
 * reallocated on demand. Invalidates the last forward's state and every
 * bsx_render_out pointer. */
BSX_API bsx_status bsx_trim(bsx_ctx* ctx);
BSX_API bsx_status bsx_sync(bsx_ctx* ctx);
BSX_API const char* bsx_last_error(const bsx_ctx* ctx);
BSX_API const char* bsx_status_string(bsx_status s);
BSX_API int bsx_abi_version(void);
/* Number of kernel launches this context has enqueued since creation. */
BSX_API uint64_t bsx_launch_count(const bsx_ctx* ctx);

/* Optional per-launch timing with CUDA events on the context's stream.
 * While enabled, every kernel launch is bracketed by two events;
 * bsx_profile_collect synchronises the stream and accumulates the elapsed
 * time per kernel name; entries are read with bsx_profile_entry. */
BSX_API bsx_status bsx_profile_enable(bsx_ctx* ctx, int32_t on);
BSX_API bsx_status bsx_profile_collect(bsx_ctx* ctx);
BSX_API int32_t bsx_profile_count(const bsx_ctx* ctx);
BSX_API bsx_status bsx_profile_entry(const bsx_ctx* ctx, int32_t i, const char** name, double* total_ms,
                                     uint64_t* launches);
BSX_API bsx_status bsx_profile_reset(bsx_ctx* ctx);

/* Host-only: camera -> uniforms, following crates/brush-render/src/camera.rs:49-101,200-254
 * and render.rs:116-136. Needs no GPU. */
BSX_API bsx_status bsx_make_project_uniforms(const bsx_camera* cam, uint32_t img_w, uint32_t img_h,
                                     uint32_t sh_degree, uint32_t total_splats,
                                     bsx_project_uniforms* out);

/* ---- forward render: SplatOps::render (crates/brush-render/src/lib.rs:69-88) ---- */
BSX_API bsx_status bsx_render_fwd(bsx_ctx* ctx, const bsx_camera* cam, uint32_t img_w, uint32_t img_h,
                          const float* d_transforms, const float* d_sh_coeffs,
                          const float* d_raw_opac, uint32_t num_splats, uint32_t sh_coeffs_per_splat,
                          int32_t render_mode, int32_t raster_pass, const float background[3],
                          bsx_render_out* out);

/* ---- backward: SplatBwdOps (crates/brush-render-bwd/src/burn_glue.rs:80-172) ----
 * Both consume the state of the last backward-pass forward render on ctx,
 * including its splat buffers (transforms, SH, opacities), which must stay
 * valid and unchanged until the backward has run. */
/* rasterize_bwd: v_output [H,W,4] -> d_v_combined [N, BSX_GRAD_STRIDE]
 * (zeroed, then accumulated). Both buffers 16-byte aligned. */
BSX_API bsx_status bsx_rasterize_bwd(bsx_ctx* ctx, const float* d_v_output, int32_t compute_refine_weight,
                             float* d_v_combined);
/* project_bwd: d_v_combined -> dense gradients (all N rows written). */
BSX_API bsx_status bsx_project_bwd(bsx_ctx* ctx, const float* d_v_combined, float* d_v_transforms,
                           float* d_v_sh_coeffs, float* d_v_raw_opac, float* d_v_refine_weight);

/* The same two operators with the reference's signatures and layouts, for a
 * backend that keeps its own forward state: stateless, compact-indexed.
 *   projected   [V,10]  rows by compact id (depth rank): xy, conic (c00 c01 c11),
 *                       opacity, rgb, depth (crates/brush-render/src/kernels/helpers.rs:48-52)
 *   compact_gid_from_isect [M] compact ids, tile-major, front to back
 *   tile_offsets [ty,tx,2] start/end per tile as the backward-pass forward left them
 *   v_combined  [V,11]  xy(2) conic(3) rgb(3) alpha refine depth
 *   global_from_compact_gid [V] splat row of each compact id
 * bsx_rasterize_bwd_ref replaces SplatBwdOps::rasterize_bwd and
 * rasterize_bwd_with_refine_weight (crates/brush-render-bwd/src/burn_glue.rs:84-121):
 * d_v_combined is zeroed, then accumulated; compute_refine_weight = 1 is
 * rasterize_bwd. render_depth = 1 returns BSX_ERR_UNSUPPORTED (depth rendering
 * is not built). out_img / v_output [H,W,4] must be 16-byte aligned.
 * bsx_project_bwd_ref replaces SplatBwdOps::project_bwd (burn_glue.rs:127-141) and
 * writes all N rows of the dense gradients (zeros for splats without a compact id).
 * An intersection id >= V, a tile range beyond M or a global id >= N is skipped
 * and reported as BSX_ERR_INVALID_ARG by the next bsx_sync (the reference's
 * checked launches skip out-of-bounds accesses the same way). Workspace: one
 * [V+1,12] row copy, the checked ids and ranges, and [max(V+1,N),12] gradient rows. */
BSX_API bsx_status bsx_rasterize_bwd_ref(bsx_ctx* ctx, const float* d_out_img, const float* d_projected,
                                         uint32_t num_visible, const uint32_t* d_compact_gid_from_isect,
                                         uint32_t num_intersections, const uint32_t* d_tile_offsets,
                                         const float background[3], uint32_t img_w, uint32_t img_h,
                                         const float* d_v_output, int32_t smooth_cutoff,
                                         int32_t compute_refine_weight, int32_t render_depth, float* d_v_combined);
BSX_API bsx_status bsx_project_bwd_ref(bsx_ctx* ctx, const float* d_transforms, const float* d_sh_coeffs,
                                       const float* d_raw_opac, uint32_t num_splats, uint32_t sh_coeffs_per_splat,
                                       const uint32_t* d_global_from_compact_gid, uint32_t num_visible,
                                       const bsx_project_uniforms* uniforms, int32_t render_mode,
                                       const float* d_v_combined, float* d_v_transforms, float* d_v_sh_coeffs,
                                       float* d_v_raw_opac, float* d_v_refine_weight);

/* ---- image loss: LossOps (crates/brush-loss/src/lib.rs:955-970) ----
 * pred/map/dl_dpred are [C,H,W] planar like the reference (C = 3, or 4 with
 * alpha matching in channel 3). */
BSX_API bsx_status bsx_loss_fwd(bsx_ctx* ctx, const float* d_pred, const uint32_t* d_gt_packed, uint32_t img_w,
                        uint32_t img_h, uint32_t channels, const bsx_loss_cfg* cfg, float* d_loss_map);
BSX_API bsx_status bsx_loss_bwd(bsx_ctx* ctx, const float* d_pred, const uint32_t* d_gt_packed, uint32_t img_w,
                        uint32_t img_h, uint32_t channels, const bsx_loss_cfg* cfg,
                        const float* d_dl_dmap, float* d_dl_dpred);
/* Fused training form: reads the [H,W,4] render directly, writes mean(map)
 * over the 3 colour channels to d_loss_mean (one float) and the gradient of
 * that mean into d_v_output [H,W,4] (alpha lane 0). */
BSX_API bsx_status bsx_loss_fused(bsx_ctx* ctx, const float* d_image_hwc4, const uint32_t* d_gt_packed,
                          uint32_t img_w, uint32_t img_h, const bsx_loss_cfg* cfg, float* d_loss_mean,
                          float* d_v_output);

/* ---- optimizer: AdamScaled (crates/brush-train/src/adam_scaled.rs:216-309) ---- */
BSX_API bsx_status bsx_adam_step(bsx_ctx* ctx, const bsx_adam_group* groups, int32_t num_groups,
                         const bsx_adam_cfg* cfg);

/* ---- data-parallel exchange over peer memory (one process per GPU) ------
 * The reference trains on one device (crates/brush-process/src/train_stream.rs:449-465,
 * crates/brush-train/src/train.rs:619-1182); these entry points are this
 * library's addition for N GPUs of one node, where each rank trains its own
 * view and the update uses the mean of the ranks' gradients.
 *
 * bsx_peer_alloc exports device memory that the other ranks' processes map
 * with bsx_peer_open (CUDA IPC; loads and stores then cross NVLink). The
 * handle is an opaque blob of BSX_PEER_HANDLE_BYTES to pass between processes.
 * An exporter frees its buffer only after every importer has closed it. */
#define BSX_MAX_RANKS 8
#define BSX_PEER_HANDLE_BYTES 64
#define BSX_DP_FLAG_WORDS 64
BSX_API bsx_status bsx_peer_alloc(bsx_ctx* ctx, uint64_t bytes, void** d_ptr, uint8_t* handle_out);
BSX_API bsx_status bsx_peer_free(bsx_ctx* ctx, void* d_ptr);
BSX_API bsx_status bsx_peer_open(bsx_ctx* ctx, const uint8_t* handle, void** d_ptr);
BSX_API bsx_status bsx_peer_close(bsx_ctx* ctx, void* d_ptr);

typedef struct bsx_dp_group {
    float* d_param[BSX_MAX_RANKS];       /* every rank's copy of the parameter [rows, cols] (own + mapped) */
    const float* d_grad[BSX_MAX_RANKS];  /* every rank's gradient [rows, cols] (own + mapped) */
    float* d_param_mc;                   /* multicast form (both non-NULL): NVLink multicast addresses of */
    const float* d_grad_mc;              /* every rank's d_param / dense d_grad buffers (NVSwitch, NVLS) */
    float* d_m;                          /* this rank's first moment for its shard rows [shard_rows, cols] */
    float* d_v;                          /* [shard_rows, cols], or [shard_rows] when reduce_moment_2 */
    uint32_t rows, cols;                 /* full parameter shape; cols <= 80 */
    float lr;
    const float* h_col_scale;            /* may be NULL (all ones); at most 80 entries */
    int32_t reduce_moment_2;
} bsx_dp_group;

typedef struct bsx_dp_exchange {
    int32_t rank, world;                 /* 1 <= world <= BSX_MAX_RANKS */
    uint32_t* d_flags[BSX_MAX_RANKS];    /* every rank's BSX_DP_FLAG_WORDS words, zeroed before the first call */
    float* d_refine[BSX_MAX_RANKS];      /* optional [refine_rows] per rank, MAX-combined in place (NULL: none) */
    uint32_t refine_rows;
    uint32_t epoch;                      /* 1, 2, 3, ... one per call, equal on every rank */
    uint64_t timeout_ns;                 /* bound on each wait for the other ranks (0: 5 s) */
    uint32_t grad_slot_rows;             /* 0: d_grad[q] is rank q's dense gradient [rows, cols].
                                          * > 0 (a multiple of 4, >= every shard's rows): d_grad[rank]
                                          * holds world slots of this rank's shard, the gradient of
                                          * rank s for shard row i at row s * grad_slot_rows + i
                                          * (filled by the ranks themselves; see bsx_train_step_dp) */
    float* d_gate[BSX_MAX_RANKS];        /* optional [gate_rows] per rank, MAX-combined in place like
                                          * d_refine (the mean-noise visibility gate; NULL: none) */
    uint32_t gate_rows;
    float* d_refine_mc;                  /* multicast form: multicast addresses of d_refine / d_gate */
    float* d_gate_mc;
} bsx_dp_exchange;

/* Multicast form (every group's d_param_mc and d_grad_mc set; grad_slot_rows 0):
 * the buffers of all ranks are bound to one NVLink multicast object each, at
 * the same offset, and the *_mc pointers are its mapping on this rank. The
 * owner of a shard then reads the ranks' summed gradient rows with one
 * in-switch reduction (multimem.ld_reduce.add) instead of a load per rank, and
 * writes each updated row once for all ranks (multimem.st), so each GPU's
 * links carry about S per direction per step (S = the parameter bytes) instead
 * of 2 (world - 1) / world S. Refine weights and gates (non-negative) take the
 * in-switch maximum of their bit patterns. The ranks' sums are formed by the
 * switch, whose order of additions is not specified; every rank still receives
 * the same rows. */
/* One kernel in place of "all-reduce the gradients, then bsx_adam_step": rank
 * r owns rows [rows*r/world, rows*(r+1)/world) of every group. After every
 * rank has arrived (a flag barrier), it sums its rows' gradients over all
 * ranks in rank order (peer loads), scales by cfg->grad_scale, applies
 * AdamScaled with its shard's moments, and stores the new rows into every
 * rank's parameters (peer stores); refine rows take the MAX over ranks the
 * same way. The launch completes only after every rank has finished reading
 * and writing, so the next step may overwrite gradients and read parameters.
 * Every rank calls it with the same epoch, groups and cfg; the result is
 * bit-identical on every rank. A wait that exceeds timeout_ns ends the launch
 * and the next bsx_sync / render readback returns BSX_ERR_DEVICE_TIMEOUT. */
BSX_API bsx_status bsx_dp_adam_step(bsx_ctx* ctx, const bsx_dp_exchange* ex, const bsx_dp_group* groups,
                                    int32_t num_groups, const bsx_adam_cfg* cfg);

/* ---- whole training step: SplatTrainer::step (crates/brush-train/src/train.rs:619-1182) ----
 * A trainer owns what one step needs besides the splats: the loss gradient
 * image, the raster-backward rows, the dense gradients (or caller-supplied
 * buffers), the AdamScaled moments, the learning-rate schedules and the
 * refine statistics. One bsx_train_step = backward-pass render -> fused
 * SSIM+L1 loss and its gradient -> raster backward -> projection backward ->
 * fused AdamScaled over transforms / SH / opacity with the reference's rate
 * table (train.rs:964-1051) -> refine statistics (stats.rs:111-121) -> the
 * mean-noise injection (train.rs:1095-1169, see mean_noise), all on the
 * context's stream. */
typedef struct bsx_train_config {        /* TrainConfig subset (crates/brush-train/src/config.rs:15-136) */
    uint32_t total_train_iters;          /* 30000 */
    double lr_mean, lr_mean_end;         /* 2e-5, 2e-7 (scaled by median_scale) */
    double lr_coeffs_dc;                 /* 2e-3 */
    float lr_coeffs_sh_scale;            /* 10: higher SH bands use lr_coeffs_dc / this */
    double lr_opac;                      /* 0.012 */
    double lr_scale, lr_scale_end;       /* 7e-3, 5e-3 */
    double lr_rotation;                  /* 2e-3 */
    float ssim_weight;                   /* 0.2: loss = (1-w) L1 + w (1 - SSIM) */
    float background[3];
    float median_scale;                  /* BoundingBox::median_size of the initial means */
    float uniform_lr;                    /* > 0: this rate for every parameter, no schedule */
    int32_t render_mode;                 /* bsx_render_mode */
    int32_t gather_stats;                /* 1: keep the RefineRecord statistics */
    /* Mean-noise injection after AdamScaled (train.rs:1095-1169; on by default in
     * the reference). Each splat's mean moves by clamp(n * w * lr_mean *
     * mean_noise_weight, +-median_scale), n ~ N(0,1) per coordinate, w =
     * clamp((1 - opacity)^150, 0, 1) times a visibility gate: with noise_vis_gate
     * (the reference's default mrnf_noise_injection) the RefineRecord visibility
     * accumulated since the last refine (this step's visible[] when gather_stats
     * is off), otherwise this step's visible[]; skipped unless median_scale is
     * finite and positive. The normals come from a counter-based generator
     * (SplitMix64 of noise_seed, the optimizer step and the splat index, Box-Muller),
     * so a step is reproducible and equal on every data-parallel rank. */
    int32_t mean_noise;                  /* 1: inject */
    int32_t noise_vis_gate;              /* 1: accumulated visibility (mrnf_noise_injection), 0: this step's */
    float mean_noise_weight;             /* 50 */
    uint64_t noise_seed;
    /* 1: also sum, over the steps a splat is visible, the norm of its screen-space
     * mean gradient in normalised device units (|d loss / d xy_pixels * (W/2, H/2)|),
     * the signal of BSX_REFINE_GRAD_THRESHOLD (bsx_trainer_grad2d_accum) */
    int32_t accumulate_grad2d;
} bsx_train_config;

typedef struct bsx_train_stats {
    uint32_t num_visible, num_intersections;
    float lr_mean;                       /* mean learning rate used by this step */
    uint32_t step;                       /* optimizer steps taken, this one included */
} bsx_train_stats;

/* Every rank's splats and gradients for bsx_train_step_dp (own + mapped). */
typedef struct bsx_dp_splats {
    float* d_transforms[BSX_MAX_RANKS];
    float* d_sh_coeffs[BSX_MAX_RANKS];
    float* d_raw_opac[BSX_MAX_RANKS];
    float* d_v_transforms[BSX_MAX_RANKS];
    float* d_v_sh_coeffs[BSX_MAX_RANKS];
    float* d_v_raw_opac[BSX_MAX_RANKS];
    /* multicast addresses of the six buffers above (all NULL: no multicast);
     * with them each rank writes its dense gradient and the exchange takes the
     * multicast form (see bsx_dp_adam_step) */
    float* mc_transforms;
    float* mc_sh_coeffs;
    float* mc_raw_opac;
    float* mc_v_transforms;
    float* mc_v_sh_coeffs;
    float* mc_v_raw_opac;
} bsx_dp_splats;

typedef struct bsx_trainer bsx_trainer;
BSX_API bsx_status bsx_trainer_create(bsx_ctx* ctx, uint32_t num_splats, uint32_t sh_coeffs_per_splat,
                                      const bsx_train_config* cfg, bsx_trainer** out);
BSX_API bsx_status bsx_trainer_destroy(bsx_trainer* tr);
/* RefineRecord arrays [N] (refine_weight_norm MAX, vis_weight SUM, max_screen_size MAX),
 * zeroed at creation; valid while the trainer lives. */
BSX_API bsx_status bsx_trainer_stats_buffers(bsx_trainer* tr, float** d_refine_weight_norm, float** d_vis_weight,
                                             float** d_max_screen_size);
/* The view-space gradient-norm sum [N] (accumulate_grad2d); zeroed with the record. */
BSX_API bsx_status bsx_trainer_grad2d_accum(bsx_trainer* tr, float** d_grad2d_accum);
/* Dense gradients of the last step ([N,10], [N,C,3], [N], refine weight [N]).
 * bsx_train_step applies AdamScaled inside the projection backward, so it
 * writes the dense gradients only after bsx_trainer_keep_gradients(tr, 1);
 * the refine weight is always written. */
BSX_API bsx_status bsx_trainer_keep_gradients(bsx_trainer* tr, int32_t on);
BSX_API bsx_status bsx_trainer_grad_buffers(bsx_trainer* tr, float** d_v_transforms, float** d_v_sh_coeffs,
                                            float** d_v_raw_opac, float** d_v_refine_weight);
/* The raster-backward rows of the last step, [N, BSX_GRAD_STRIDE] by global id
 * (the input of its projection backward); valid until the next step. */
BSX_API bsx_status bsx_trainer_raster_grads(bsx_trainer* tr, float** d_v_combined);
/* One step in place on the splats. d_loss receives the step's mean loss (one float, device). */
BSX_API bsx_status bsx_train_step(bsx_trainer* tr, const bsx_camera* cam, uint32_t img_w, uint32_t img_h,
                                  const uint32_t* d_gt_packed, float* d_transforms, float* d_sh_coeffs,
                                  float* d_raw_opac, int32_t compute_refine_weight, float* d_loss,
                                  bsx_train_stats* stats);
/* Data-parallel step: this rank renders its view from its own copy of the
 * splats, writes its gradients and ex->d_refine[rank], then bsx_dp_adam_step
 * (gradient scale 1/world) updates every rank's copy. With
 * ex->grad_slot_rows > 0 the buffers sp->d_v_*[q] hold world * grad_slot_rows
 * rows and the projection backward stores each gradient row straight into
 * slot `rank` of the row's owner (peer stores overlapped with its compute),
 * so the exchange reads only local memory; otherwise, and after
 * bsx_trainer_keep_gradients(tr, 1), sp->d_v_*[rank] receives this rank's
 * dense gradient and the exchange pulls the peers' rows.
 * The trainer numbers the exchange epochs itself (ex->epoch is ignored), so
 * every rank's trainer must take the same data-parallel steps on flag words
 * that no other exchange uses. */
BSX_API bsx_status bsx_train_step_dp(bsx_trainer* tr, const bsx_camera* cam, uint32_t img_w, uint32_t img_h,
                                     const uint32_t* d_gt_packed, const bsx_dp_exchange* ex,
                                     const bsx_dp_splats* sp, int32_t compute_refine_weight, float* d_loss,
                                     bsx_train_stats* stats);

/* ---- densification: SplatTrainer::refine_for_phase (crates/brush-train/src/train.rs:1191-1534) ----
 * Two calls, because the splat count changes:
 *   bsx_trainer_refine_plan decides, from the splats and the trainer's
 *   RefineRecord: the prune mask (opacity, oversize, out-of-bounds, non-finite,
 *   tiny scale, degenerate rotation; train.rs:1268-1350), the replacement of
 *   pruned splats (weighted by opacity x visibility), the forced split of
 *   splats too large on screen, and gradient-threshold growth; it returns the
 *   new count in stats->total_splats.
 *   bsx_trainer_refine_apply writes the refined splats into caller buffers of
 *   that count (kept rows in order, then one child per split splat), applies
 *   the long-axis split (train.rs:1547-1700) and the opacity / scale decay
 *   (train.rs:1700-1740), compacts and zeroes the Adam moments as the
 *   reference does, resets the RefineRecord and resizes the trainer.
 * Sampling: weighted sampling without replacement (the reference's
 * rand::seq::index::sample_weighted, crates/brush-train/src/multinomial.rs),
 * realised with Efraimidis-Spirakis keys log(u)/w from a counter-based
 * generator (SplitMix64 of seed, refine count and index): deterministic, and
 * the same distribution as the reference's, not the same draws. The growth
 * signal is the gradient norm (error-map / edge-map growth are not built). */
/* Densification rules:
 *   BSX_REFINE_REFERENCE: the reference's refine_for_phase (above).
 *   BSX_REFINE_GRAD_THRESHOLD: the gradient-threshold rule of the original 3D
 *   Gaussian splatting trainer (Kerbl et al. 2023, densify_and_clone /
 *   densify_and_split / prune), which the densification benchmark describes:
 *   after the same prune mask, every kept splat whose view-space gradient norm
 *   averaged over its visible steps (grad2d_accum / vis_weight) is at least
 *   growth_grad_threshold is cloned (a copy appended) when its largest scale is
 *   at most percent_dense times the largest bounds extent, else split: it is
 *   replaced by two children at mean + R (s * n), n ~ N(0,1)^3 from the
 *   counter-based generator, with scales s / 1.6 and the other parameters
 *   copied. New rows have zero Adam moments; no opacity or scale decay. Rows:
 *   kept splats that are not split (in order), clones, first children, second
 *   children; clones then splits are cut to max_splats in row order. Needs a
 *   trainer with accumulate_grad2d. */
#define BSX_REFINE_REFERENCE 0
#define BSX_REFINE_GRAD_THRESHOLD 1
typedef struct bsx_refine_config {       /* refine options (crates/brush-train/src/config.rs:100-330) */
    uint32_t max_splats;                 /* 10,000,000 */
    float growth_grad_threshold;         /* 0.0025 */
    float growth_select_fraction;        /* 0.07 */
    uint32_t growth_stop_iter;           /* 15000 */
    float split_at_screen_size;          /* 0.5 (0 disables) */
    float opac_decay;                    /* 0.004 */
    float scale_decay;                   /* 0.002 */
    int32_t min_scale_prune;             /* 1 */
    float min_scale_prune_threshold;     /* 1e-10 */
    int32_t near_zero_rotation_prune;    /* 1 */
    int32_t radial_bounds_prune;         /* 0: per-axis (L-inf) bounds test */
    float min_opacity;                   /* 1/255 */
    float prune_extent_factor;           /* 100 */
    float split_long_axis_scale;         /* 0.5 */
    float split_other_axis_scale;        /* 0.85 */
    float split_opacity_scale;           /* 0.6 */
    uint64_t seed;
    int32_t rule;                        /* BSX_REFINE_REFERENCE or BSX_REFINE_GRAD_THRESHOLD */
    float percent_dense;                 /* 0.01: clone / split boundary (gradient-threshold rule) */
} bsx_refine_config;

typedef struct bsx_refine_stats {        /* RefineStats (train.rs:1520-1530) */
    uint32_t num_added, num_split_oversized, num_split_high_grad;
    uint32_t num_pruned, num_pruned_non_finite, total_splats;
} bsx_refine_stats;

/* bounds_center / bounds_extent: the trainer's current BoundingBox (percentile
 * bounds of the means, splat_init.rs:130-158); max_allowed = max extent *
 * prune_extent_factor. */
BSX_API bsx_status bsx_trainer_refine_plan(bsx_trainer* tr, const float* d_transforms, const float* d_sh_coeffs,
                                           const float* d_raw_opac, const bsx_refine_config* cfg,
                                           const float bounds_center[3], const float bounds_extent[3],
                                           uint32_t global_iter, bsx_refine_stats* stats);
BSX_API bsx_status bsx_trainer_refine_apply(bsx_trainer* tr, const float* d_transforms, const float* d_sh_coeffs,
                                            const float* d_raw_opac, float* d_new_transforms, float* d_new_sh_coeffs,
                                            float* d_new_raw_opac, uint32_t phase_iter, uint32_t phase_total);
/* The AdamScaled moments (first m, second v) per group and the rows they cover;
 * NULL pointers before the first optimizer step. v of the SH group is per row. */
BSX_API bsx_status bsx_trainer_optimizer_state(bsx_trainer* tr, float** d_m_transforms, float** d_m_sh_coeffs,
                                               float** d_m_raw_opac, float** d_v_transforms, float** d_v_sh_coeffs,
                                               float** d_v_raw_opac, uint32_t* rows);
/* Allocate now every buffer the trainer and its context index by splat, for
 * up to max_splats splats (gradients, moments, statistics, refine scratch,
 * projected rows, counts and ids), so a growing run does not allocate at its
 * refines. Buffers sized by intersections still grow on demand. */
BSX_API bsx_status bsx_trainer_reserve(bsx_trainer* tr, uint32_t max_splats);
/* Replace the moments with the given rows: the whole model (world 1), or the
 * shard rows [rows_total*rank/world, rows_total*(rank+1)/world) the
 * data-parallel step of `rank` of `world` uses, where rows_total is the
 * trainer's splat count. Device arrays laid out as bsx_trainer_optimizer_state
 * returns them; the Adam time step is kept. */
BSX_API bsx_status bsx_trainer_load_optimizer_state(bsx_trainer* tr, const float* d_m_transforms,
                                                    const float* d_m_sh_coeffs, const float* d_m_raw_opac,
                                                    const float* d_v_transforms, const float* d_v_sh_coeffs,
                                                    const float* d_v_raw_opac, uint32_t rows, int32_t world,
                                                    int32_t rank);
/* The trainer's bounding box: bounds_from_pos (crates/brush-train/src/splat_init.rs:130-158).
 * Per axis the order statistics trunc(f32((1 - p) / 2) * n) and
 * min(n - 1, trunc(f32((1 + p) / 2) * n)) of the n finite coordinates under
 * total_cmp, then center = (max + min) / 2, extent = (max - min) / 2
 * (BoundingBox::from_min_max); no finite coordinate on some axis: [-1, 1]^3.
 * d_means: N rows of `stride` floats whose first three are the mean (stride 10
 * for a transforms tensor). Synchronises the context's stream. */
BSX_API bsx_status bsx_splat_bounds(bsx_ctx* ctx, const float* d_means, uint32_t stride, uint32_t num_splats,
                                    float percentile, float center[3], float extent[3]);
/* Rate schedule input after the bounds change (train.rs:656: lr_mean uses bounds.median_size()). */
BSX_API bsx_status bsx_trainer_set_median_scale(bsx_trainer* tr, float median_scale);

/* The mean-noise step of SplatTrainer::step_with_refine_weight (train.rs:1095-1169)
 * as an operator, in place on the means of d_transforms [N,10]: for splat i with
 * d_gate[i] > 0, mean += clamp(n * w * scale, -limit, limit), n ~ N(0,1) from
 * (seed, step, i) as bsx_train_config describes, w = clamp((1 -
 * sigmoid(d_raw_opac[i]))^150, 0, 1), scale = f32(lr_mean) * mean_noise_weight,
 * limit = the median bounds size. The trainer applies the same arithmetic inside
 * its step; this entry point serves steps composed from the operators. */
BSX_API bsx_status bsx_mean_noise_step(bsx_ctx* ctx, float* d_transforms, const float* d_raw_opac,
                                       const float* d_gate, uint32_t num_splats, float scale, float limit,
                                       uint64_t seed, uint32_t step);

/* ---- primitives: brush-sort / brush-prefix-sum / get_tile_offsets ---- */
/* Stable argsort by key & mask(bits rounded up to a multiple of 4), as
 * crates/brush-sort/src/lib.rs:16-129. Inputs are left untouched. */
BSX_API bsx_status bsx_radix_argsort_u32(bsx_ctx* ctx, const uint32_t* d_keys, const uint32_t* d_values, uint32_t n,
                                 uint32_t sorting_bits, uint32_t* d_keys_out, uint32_t* d_values_out);
/* Inclusive prefix sum (u32, wrapping), crates/brush-prefix-sum/src/lib.rs:11-87. */
BSX_API bsx_status bsx_prefix_sum_u32(bsx_ctx* ctx, const uint32_t* d_in, uint32_t n, uint32_t* d_out);
/* Allocation-free variant of bsx_prefix_sum_u32 (no counterpart in the
 * reference: an addition of this library for callers that cannot allocate GPU
 * memory, e.g. inside a foreign memory pool, in a real-time loop that cannot
 * afford cudaMalloc's synchronisation, or in a host that does not let a plugin
 * create a context). Same result as bsx_prefix_sum_u32; runs on the current
 * device and the given stream, which must belong to the current device
 * (BSX_ERR_INVALID_ARG otherwise); needs no context. Its scratch is one fixed
 * device array per GPU (32 KiB, resident until exit) shared by all calls:
 * calls that overlap on the GPU race, so serialise them. n is limited to
 * BSX_PREFIX_SUM_NOALLOC_MAX_N (BSX_ERR_CAPACITY beyond). The first call on a
 * device resolves the array's address and should precede any stream capture. */
#define BSX_PREFIX_SUM_NOALLOC_MAX_N 16769024u
BSX_API bsx_status bsx_prefix_sum_u32_noalloc(const uint32_t* d_in, uint32_t n, uint32_t* d_out, void* cuda_stream);
/* [start,end) per tile from sorted tile ids; ids >= num_tiles are sentinels
 * (crates/brush-render/src/get_tile_offset.rs:10-62). d_offsets is zeroed first. */
BSX_API bsx_status bsx_get_tile_offsets(bsx_ctx* ctx, const uint32_t* d_tile_ids, uint32_t n, uint32_t num_tiles,
                                uint32_t* d_offsets);

/* ---- splat PLY import / export (crates/brush-serde) ----
 * bsx_ply_parse reads the header and the row layout of a PLY byte buffer
 * (ascii, binary_little_endian or binary_big_endian; the standard 3DGS vertex
 * properties, or the SuperSplat compressed chunk/vertex/sh layout), validates
 * it as stream_splat_from_ply does (crates/brush-serde/src/import.rs:180-333)
 * and keeps every subsample-th row. It needs no GPU. On BSX_ERR_FORMAT, err
 * receives the reason (the reference's messages). For little-endian binary
 * input the parsed file refers to `bytes`, which must stay valid and unchanged
 * until the stream has executed bsx_ply_load.
 * bsx_ply_load decodes on the device into the splat layout: transforms
 * [N,10] (mean, quaternion w x y z, log-scale), sh [N, sh_coeffs, 3]
 * (coefficient-major) and raw opacities [N], N = info.num_splats. Absent
 * fields take the reference's defaults (import.rs:77-95).
 * bsx_ply_export writes splat_to_ply's file (crates/brush-serde/src/export.rs:
 * 84-191: binary little-endian, quaternion normalised, SH rest in the
 * channel-major order of the 3DGS format) into host memory; up_axis may be
 * NULL ("Vertical axis: y"). It synchronises the context's stream. */
typedef struct bsx_ply_info {
    uint32_t num_splats;   /* rows kept after subsampling */
    uint32_t total_rows;   /* vertex rows in the file */
    uint32_t sh_coeffs;    /* SH coefficients per channel of the decoded splats */
    uint32_t subsample;
    int32_t compressed;    /* SuperSplat compressed layout */
    int32_t render_mode;   /* -1 none, 0 default, 1 mip ("SplatRenderMode:" comment) */
    int32_t has_up_axis;   /* "Vertical axis:" comment */
    float up_axis[3];
} bsx_ply_info;
typedef struct bsx_ply_file bsx_ply_file;
BSX_API bsx_status bsx_ply_parse(const uint8_t* bytes, size_t len, uint32_t subsample, bsx_ply_file** out,
                                 bsx_ply_info* info, char* err, size_t err_len);
BSX_API void bsx_ply_free(bsx_ply_file* f);
BSX_API bsx_status bsx_ply_load(bsx_ctx* ctx, const bsx_ply_file* f, float* d_transforms, float* d_sh,
                                float* d_raw_opac);
BSX_API bsx_status bsx_ply_export_size(uint32_t n, uint32_t sh_coeffs, int32_t mip, const float* up_axis,
                                       uint64_t* bytes);
BSX_API bsx_status bsx_ply_export(bsx_ctx* ctx, const float* d_transforms, const float* d_sh,
                                  const float* d_raw_opac, uint32_t n, uint32_t sh_coeffs, int32_t mip,
                                  const float* up_axis, uint8_t* host_out, uint64_t capacity, uint64_t* written);

#ifdef __cplusplus
}
#endif
#endif /* BSX_H */
