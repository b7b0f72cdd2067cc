// common.cuh - internal definitions shared by the bsx CUDA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/bsx.h"
#include "../../include/bsx_fmath.h"

namespace bsx {

// Row stride of the raster-backward gradient buffer: the 11 reference lanes
// plus one pad lane so each row is three 16-byte words (vector atomics).
constexpr int kGradStride = 12;
constexpr int kTile = BSX_TILE_WIDTH;
constexpr int kTilePixels = kTile * kTile;

// Device error word codes (first writer wins).
enum DeviceError : int {
    kDevOk = 0,
    kDevLookbackTimeout = 1,
    kDevOutOfRange = 2,
    kDevPeerTimeout = 3,
    kDevBadIndex = 4,  // a caller-supplied index or range was out of bounds (entry skipped)
};

// Bounded spin for device-side waits on another block's published state.
// A block that gives up records kDevLookbackTimeout and proceeds with a
// (wrong but finite) value so that the grid always terminates.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ void set_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// System-scope flag accesses for waits on other GPUs (peer memory over NVLink).
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// AdamScaled applied inside the projection backward (single-GPU trainer): the
// moments, rates and per-column scales of the three parameter groups, with
// the same arithmetic as bsx_adam_step (adam.cu).
struct FusedAdam {
    float* m_t;   // [N,10]
    float* m_sh;  // [N,3C]
    float* m_o;   // [N]
    float* v_t;   // [N,10]
    float* v_sh;  // [N] (second moment per row)
    float* v_o;   // [N]
    float lr_t, lr_sh, lr_op;
    int has_t_scale, has_sh_scale;
    float t_scale[10];
    float sh_scale[80];
    float b1, b2, eps, inv_bc1, inv_bc2, gscale;
    int first;
    int keep_grads;  // also write the dense gradients
};

// Data-parallel gradient push from the projection backward. Rank q owns rows
// [n q / world, n (q + 1) / world); owner q's gradient region of group k
// (transforms, SH rows, opacities) holds `world` slots of its shard, and the
// gradient that rank s computed for global row g (owned by q) goes to
// dst[k][q] + (s * slot_rows + g - shard_begin(q)) * cols. world == 0: no push.
struct GradPush {
    float* dst[3][BSX_MAX_RANKS];
    uint32_t n, slot_rows;
    int world, rank;
};

__host__ __device__ inline uint32_t shard_begin(uint32_t n, int q, int world) {
    return (uint32_t)((uint64_t)n * (uint32_t)q / (uint32_t)world);
}
// Owner of row g: floor(g world / n) never exceeds it and is at most one below.
__host__ __device__ inline int shard_owner(uint32_t n, uint32_t g, int world) {
    int q = (int)(((uint64_t)g * (uint32_t)world) / n);
    if (q + 1 < world && shard_begin(n, q + 1, world) <= g) ++q;
    return q;
}

// 1 / (1 - beta^step) in float, by repeated multiplication (adam.cu fill_cfg).
inline float adam_inv_bias_correction(float beta, uint32_t step) {
    float r = 1.0f;
    for (uint32_t i = 0; i < step; ++i) r *= beta;
    return 1.0f / (1.0f - r);
}

// Grow-only device buffer owned by a context.
struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};

}  // namespace bsx

// Forward-render state kept for the backward entry points
// (mirrors GaussianBackwardState, crates/brush-render-bwd/src/burn_glue.rs:264-284).
struct bsx_fwd_state {
    int valid = 0;
    int bwd_info = 0;
    int smooth = 0;
    int mip = 0;
    uint32_t n = 0, coeffs = 0, degree = 0;
    uint32_t num_visible = 0, num_intersections = 0;
    float bg[3] = {0, 0, 0};
    bsx_project_uniforms uni{};
    const float* transforms = nullptr;
    const float* sh = nullptr;
    const float* raw_opac = nullptr;
};

struct bsx_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string last_error;
    uint64_t launches = 0;
    int* d_err = nullptr;            // device error word
    uint32_t* h_pinned = nullptr;    // pinned readback slots
    // workspace
    bsx::DevBuf projected, counts, depth_keys, vis_gid, depth_order, cum, isect_tile, isect_gid, tile_offsets,
        image, image_packed, visible, max_radius, sort_tmp_k, sort_tmp_v, sort_hist, sort_lookback, scan_status,
        scalars, grad, loss_partials, loss_planes, sort_keys_b, sort_vals_b, tile_order, isect_mask,
        // reference-layout backward operators (ref_bwd.cu)
        ref_rows, ref_ids, ref_offsets, ref_grad, ref_order,
        // percentile bounds of the means (bounds.cu)
        bounds_tmp;
    bsx_fwd_state fwd;
    // optional per-launch timing (bsx_profile_*)
    int profiling = 0;
    cudaEvent_t prof_start = nullptr;
    struct ProfRec {
        const char* name;
        cudaEvent_t a, b;
    };
    std::vector<ProfRec> prof_pending;
    std::vector<cudaEvent_t> prof_pool;
    std::vector<std::string> prof_names;
    std::vector<double> prof_ms;
    std::vector<uint64_t> prof_count;
};

namespace bsx {

bsx_status fail(bsx_ctx* ctx, bsx_status s, const std::string& msg);
bsx_status check_cuda(bsx_ctx* ctx, cudaError_t e, const char* what);
bsx_status ensure(bsx_ctx* ctx, DevBuf& b, size_t bytes);
// Stream-ordered release of a workspace buffer.
void release(bsx_ctx* ctx, DevBuf& b);
// Records a start event before a kernel launch when profiling is on.
void prof_begin(bsx_ctx* ctx);
// Checks the launch that was just enqueued and counts it.
bsx_status post_launch(bsx_ctx* ctx, const char* name);
// Reads and clears the device error word (synchronises the stream).
bsx_status check_device_error(bsx_ctx* ctx);

// ---- primitives (scan.cu, sort.cu) ----
// Inclusive scan of n u32 (optionally gathered: in[gather[i]]). Writes the
// total to d_total if non-null. Uses ctx->scan_status as lookback state.
bsx_status scan_inclusive_u32(bsx_ctx* ctx, const uint32_t* d_in, const uint32_t* d_gather, uint32_t n,
                              uint32_t* d_out, uint32_t* d_total);
// Stable LSD radix argsort of (key & mask(ceil4(bits))) with u32 values.
bsx_status radix_sort_pairs(bsx_ctx* ctx, const uint32_t* d_keys, const uint32_t* d_vals, uint32_t n,
                            uint32_t bits, uint32_t* d_keys_out, uint32_t* d_vals_out);
bsx_status tile_offsets(bsx_ctx* ctx, const uint32_t* d_ids, uint32_t n, uint32_t num_tiles, uint32_t* d_off);
// Launch order of the tiles for the rasterizers (descending intersection count).
bsx_status tile_order(bsx_ctx* ctx, const uint32_t* d_off, uint32_t num_tiles, uint32_t* d_order);

// Lookback state for the scan family: per-tile status words plus a ticket.
size_t scan_status_words(uint32_t n_tiles);

}  // namespace bsx
