// project_fwd.cu - fused cull / project / SH colour, then visible compaction.
//
// project_fwd_kernel: one thread per splat, 256 splats per block. Restates, in
// one pass, project_forward_kernel (crates/brush-render/src/kernels/project_forward.rs:20-144)
// and project_visible_kernel (kernels/project_visible.rs:22-89): the cull
// predicates, the EWA covariance, the StopThePop per-tile count, and the SH
// colour of every surviving splat. The per-tile count is taken by the warp
// together (tile_walk.cuh) instead of one lane per box. No block-wide
// barrier: every block streams independently.
//
// compact_visible_kernel: where the reference appends visible ids with an
// atomic counter (order depends on scheduling), blocks of 1024 splats here
// take tickets and compact with a decoupled look-back over the projection's
// per-warp visibility masks, so the visible list is in global-id order on
// every run; the same pass sums the intersection counts.
//
// Outputs (global-id indexed unless noted):
//   projected[N,12]  rows {x, y, conic00, conic01, conic11, opacity, r, g, b,
//                    depth, ln(255*opacity), 0}; written for visible splats only
//   counts[N]        contributing-tile count (0 when culled)
//   max_radius[N]    max(ex/W, ey/H) (0 when culled)
//   vis_gid[V], depth_key[V]  compacted visible ids and depth bits, id order
//   scalars[0] = V, scalars[1] = total intersections (u32, wraps as the reference)
// Scratch: vis_mask[ceil(N/32)] (bit per splat), depth_dense[N] (visible only).
#include "lookback.cuh"
#include "sh.cuh"
#include "tile_walk.cuh"

namespace bsx {

namespace {

constexpr int kProjThreads = 256;

struct ProjArgs {
    const float* transforms;
    const float* sh;
    const float* raw_opac;
    uint32_t n;
    uint32_t coeffs;
    int mip;
    int sh_vec;  // SH base 16-byte aligned
    Uni u;
    float* projected;
    uint32_t* counts;
    float* max_radius;
    uint32_t* vis_mask;
    uint32_t* depth_dense;
};

struct CompactArgs {
    const uint32_t* vis_mask;
    const uint32_t* depth_dense;
    const uint32_t* counts;
    uint32_t n;
    uint32_t* vis_gid;
    uint32_t* depth_key;
    uint32_t* scalars;
    uint64_t* status;
    uint32_t* ticket;
    int* err;
};

// Register-bounded to four resident blocks per SM: the kernel is latency-bound
// (long dependent chains of exp / log / sqrt / division per splat), and the
// extra warps outweigh the few spilled registers of the degree-3 instance.
template <int DEG>
__global__ void __launch_bounds__(kProjThreads, 4) project_fwd_kernel(const __grid_constant__ ProjArgs a) {
    const uint32_t g = blockIdx.x * kProjThreads + threadIdx.x;
    const Uni& u = a.u;

    // Cull and project; a surviving splat leaves its tile box for the walk.
    bool visible = false;
    WalkSplat ws{0u, 0u, 0u, 0u, 0.0f, 0.0f, S2{0.0f, 0.0f, 0.0f}, 0.0f};
    V3 mean = v3(0.0f, 0.0f, 0.0f);
    float depth = 0.0f, radius = 0.0f, opac = 0.0f;
    if (g < a.n) {
        do {
            // one transform row = five 8-byte words
            const float2* t2 = reinterpret_cast<const float2*>(a.transforms + (size_t)g * 10);
            const float2 w0 = __ldg(t2), w1 = __ldg(t2 + 1), w2 = __ldg(t2 + 2), w3 = __ldg(t2 + 3), w4 = __ldg(t2 + 4);
            const float t[10] = {w0.x, w0.y, w1.x, w1.y, w2.x, w2.y, w3.x, w3.y, w4.x, w4.y};
            mean = v3(t[0], t[1], t[2]);
            V3 mean_c = vadd(mmul(u.rot, mean), u.trans);
            if (!(vfinite(mean_c) && mean_c.z <= 1.0e10f)) break;
            if (u.model == BSX_CAMERA_PINHOLE) {
                if (mean_c.z < 0.01f) break;
            } else {  // fisheye-capable models cull by the ray angle (project_forward.rs:49-64)
                const float rr = sqrtf(mean_c.x * mean_c.x + mean_c.y * mean_c.y);
                if (bsx_atan2f(rr, mean_c.z) > u.half_max_fov) break;
            }
            V3 scl = v3(bsx_expf(t[7]), bsx_expf(t[8]), bsx_expf(t[9]));
            if (!vfinite(scl)) break;
            Q4 qu{t[3], t[4], t[5], t[6]};
            float qn = qdot(qu, qu);
            if (!(qn >= 1.0e-6f && bsx_is_finite(qn))) break;
            float ro = __ldg(a.raw_opac + g);
            if (!bsx_is_finite(ro)) break;
            Q4 q = qnormalize(qu);
            S2 raw = calc_cov2d(scl, q, mean_c, u);
            float fc;
            S2 cov = compensate_cov2d(raw, a.mip != 0, &fc);
            opac = bsx_sigmoid(ro) * fc;
            if (!s2finite(cov)) break;
            float m2x, m2y;
            project_mean(mean_c, u, &m2x, &m2y);
            if (!(opac >= 1.0f / 255.0f)) break;
            float pt = bsx_logf(opac * 255.0f);
            S2 conic = sym2_inverse(cov);
            float ex, ey;
            bbox_extent(conic, pt, &ex, &ey);
            if (!(ex >= 0.0f && ey >= 0.0f)) break;
            float wf = (float)u.w, hf = (float)u.h;
            bool on_screen = m2x + ex > 0.0f && m2x - ex < wf && m2y + ey > 0.0f && m2y - ey < hf;
            if (!on_screen) break;
            TileBox bb = tile_bbox(m2x, m2y, ex, ey, u.tbw, u.tbh);
            const uint32_t bw = bb.max_x > bb.min_x ? bb.max_x - bb.min_x : 0u;
            const uint32_t bh = bb.max_y > bb.min_y ? bb.max_y - bb.min_y : 0u;
            ws = WalkSplat{bb.min_x, bb.min_y, bw, bw * bh, m2x, m2y, conic, pt};
            visible = true;
            depth = mean_c.z;
            radius = bsx_max(ex / wf, ey / hf);
        } while (false);
    }

    // The visible splat's SH row (12 C bytes) starts towards L2 now and is read
    // after the walk below.
    if (visible) {
        constexpr uint32_t kRowBytes = (DEG + 1) * (DEG + 1) * 12;
        const char* srow = reinterpret_cast<const char*>(a.sh + (size_t)g * ((DEG + 1) * (DEG + 1) * 3));
#pragma unroll
        for (uint32_t off = 0; off < kRowBytes; off += 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(srow + off));
    }

    // Contributing-tile count: the warp walks its splats' boxes together.
    uint32_t hits = 0;
    warp_tile_walk(ws, [&](const WalkStep& s) { hits += s.own; });

    if (visible) {
        // SH colour at the normalised view direction (project_visible.rs:56-71).
        V3 dv = vsub(mean, u.cam);
        V3 vdir = vscale(dv, 1.0f / sqrtf(vdot(dv, dv)));
        constexpr int C3 = (DEG + 1) * (DEG + 1) * 3;
        float shc[C3];
        const float* srow = a.sh + (size_t)g * C3;
        if (C3 % 4 == 0 && a.sh_vec) {
#pragma unroll
            for (int k = 0; k < C3 / 4; ++k) {
                const float4 q4 = __ldg(reinterpret_cast<const float4*>(srow) + k);
                shc[4 * k] = q4.x;
                shc[4 * k + 1] = q4.y;
                shc[4 * k + 2] = q4.z;
                shc[4 * k + 3] = q4.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < C3; ++k) shc[k] = __ldg(srow + k);
        }
        V3 col = sh_to_color<DEG>(shc, vdir);
        float cr = col.x + 0.5f, cg = col.y + 0.5f, cb = col.z + 0.5f;
        cr = bsx_clamp(bsx_is_finite(cr) ? cr : 0.0f, -100.0f, 100.0f);
        cg = bsx_clamp(bsx_is_finite(cg) ? cg : 0.0f, -100.0f, 100.0f);
        cb = bsx_clamp(bsx_is_finite(cb) ? cb : 0.0f, -100.0f, 100.0f);
        float4* row = reinterpret_cast<float4*>(a.projected + (size_t)g * BSX_PROJECTED_LANES);
        row[0] = make_float4(ws.mx, ws.my, ws.conic.c00, ws.conic.c01);
        row[1] = make_float4(ws.conic.c11, opac, cr, cg);
        row[2] = make_float4(cb, depth, ws.pt, 0.0f);
    }
    if (g < a.n) {
        a.counts[g] = hits;
        a.max_radius[g] = radius;
    }

    const uint32_t vmask = __ballot_sync(0xffffffffu, visible);
    if ((threadIdx.x & 31) == 0 && g < a.n) a.vis_mask[g >> 5] = vmask;
    if (visible) a.depth_dense[g] = bsx_f32_to_bits(depth);
}

constexpr int kCompactThreads = 256;
constexpr int kCompactPer = 4;  // splats per thread
constexpr uint32_t kCompactTile = kCompactThreads * kCompactPer;

// Ordered compaction of the visible ids + intersection total.
__global__ void __launch_bounds__(kCompactThreads) compact_visible_kernel(const __grid_constant__ CompactArgs a) {
    __shared__ uint32_t s_tile;
    __shared__ uint32_t s_warp_vis[kCompactThreads / 32];
    __shared__ uint32_t s_warp_hits[kCompactThreads / 32];
    __shared__ uint32_t s_base;
    if (threadIdx.x == 0) s_tile = atomicAdd(a.ticket, 1u);
    __syncthreads();
    const uint32_t tile = s_tile;
    const uint32_t g0 = tile * kCompactTile + threadIdx.x * kCompactPer;
    // 4 consecutive splats never straddle a 32-bit mask word
    const uint32_t word = g0 < a.n ? __ldg(a.vis_mask + (g0 >> 5)) : 0u;
    uint32_t bits = (word >> (g0 & 31)) & 0xfu;
    uint32_t hits = 0;
#pragma unroll
    for (int k = 0; k < kCompactPer; ++k) {
        if (g0 + k < a.n) hits += __ldg(a.counts + g0 + k);
        else bits &= ~(1u << k);
    }
    const uint32_t nvis = __popc(bits);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = nvis;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    uint32_t whits = hits;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) whits += __shfl_xor_sync(0xffffffffu, whits, o);
    if (lane == 31) s_warp_vis[warp] = inc;
    if (lane == 0) s_warp_hits[warp] = whits;
    __syncthreads();
    if (warp == 0) {
        const uint32_t wv = lane < kCompactThreads / 32 ? s_warp_vis[lane] : 0u;
        uint32_t wh = lane < kCompactThreads / 32 ? s_warp_hits[lane] : 0u;
        uint32_t winc = wv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, winc, o);
            if (lane >= o) winc += t;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wh += __shfl_xor_sync(0xffffffffu, wh, o);
        const uint32_t block_vis = __shfl_sync(0xffffffffu, winc, 31);
        if (lane < kCompactThreads / 32) s_warp_vis[lane] = winc - wv;
        const uint32_t prefix = lookback_publish(a.status, tile, block_vis, a.err);
        if (lane == 0) {
            s_base = prefix;
            if (wh) atomicAdd(a.scalars + 1, wh);
            if ((uint64_t)(tile + 1) * kCompactTile >= a.n) a.scalars[0] = prefix + block_vis;
        }
    }
    __syncthreads();
    uint32_t pos = s_base + s_warp_vis[warp] + inc - nvis;
#pragma unroll
    for (int k = 0; k < kCompactPer; ++k) {
        if (bits & (1u << k)) {
            if (pos < a.n) {
                a.vis_gid[pos] = g0 + k;
                a.depth_key[pos] = __ldg(a.depth_dense + g0 + k);
            } else {
                set_error(a.err, kDevOutOfRange);
            }
            ++pos;
        }
    }
}

}  // namespace

bsx_status launch_project_fwd(bsx_ctx* ctx, const bsx_project_uniforms& uni, const float* transforms,
                              const float* sh, const float* raw_opac, uint32_t n, uint32_t coeffs, int degree,
                              int mip, float* projected, uint32_t* counts, float* max_radius, uint32_t* vis_gid,
                              uint32_t* depth_key, uint32_t* scalars, uint32_t* vis_mask, uint32_t* depth_dense) {
    if (degree < 0 || degree > 4) return fail(ctx, BSX_ERR_SHAPE, "sh coefficient count must be (degree+1)^2 with degree <= 4");
    const uint32_t blocks = (n + kProjThreads - 1) / kProjThreads;
    const uint32_t tiles = (n + kCompactTile - 1) / kCompactTile;
    bsx_status s = ensure(ctx, ctx->scan_status, scan_status_words(tiles) * sizeof(uint64_t));
    if (s != BSX_OK) return s;
    uint64_t* status = ctx->scan_status.as<uint64_t>();
    s = check_cuda(ctx, cudaMemsetAsync(status, 0, scan_status_words(tiles) * sizeof(uint64_t), ctx->stream),
                   "memset compaction status");
    if (s != BSX_OK) return s;
    s = check_cuda(ctx, cudaMemsetAsync(scalars, 0, 2 * sizeof(uint32_t), ctx->stream), "memset scalars");
    if (s != BSX_OK) return s;
    if (n == 0) return BSX_OK;
    ProjArgs a;
    a.transforms = transforms;
    a.sh = sh;
    a.raw_opac = raw_opac;
    a.n = n;
    a.coeffs = coeffs;
    a.mip = mip;
    a.sh_vec = ((uintptr_t)sh % 16) == 0;
    a.u = make_uni(uni);
    a.projected = projected;
    a.counts = counts;
    a.max_radius = max_radius;
    a.vis_mask = vis_mask;
    a.depth_dense = depth_dense;
    prof_begin(ctx);
    switch (degree) {
        case 0: project_fwd_kernel<0><<<blocks, kProjThreads, 0, ctx->stream>>>(a); break;
        case 1: project_fwd_kernel<1><<<blocks, kProjThreads, 0, ctx->stream>>>(a); break;
        case 2: project_fwd_kernel<2><<<blocks, kProjThreads, 0, ctx->stream>>>(a); break;
        case 3: project_fwd_kernel<3><<<blocks, kProjThreads, 0, ctx->stream>>>(a); break;
        default: project_fwd_kernel<4><<<blocks, kProjThreads, 0, ctx->stream>>>(a); break;
    }
    s = post_launch(ctx, "project_fwd_kernel");
    if (s != BSX_OK) return s;
    CompactArgs c;
    c.vis_mask = vis_mask;
    c.depth_dense = depth_dense;
    c.counts = counts;
    c.n = n;
    c.vis_gid = vis_gid;
    c.depth_key = depth_key;
    c.scalars = scalars;
    c.status = status;
    c.ticket = reinterpret_cast<uint32_t*>(status + tiles);
    c.err = ctx->d_err;
    prof_begin(ctx);
    compact_visible_kernel<<<tiles, kCompactThreads, 0, ctx->stream>>>(c);
    return post_launch(ctx, "compact_visible_kernel");
}

}  // namespace bsx
