// raster_bwd.cu - tile rasterizer, backward.
//
// Restates rasterize_backwards_kernel
// (crates/brush-render-bwd/src/kernels/rasterize_backwards.rs:79-443) with a
// pixel-parallel schedule: one 128-thread block per 16x16 tile, two pixels per
// thread (Morton position (x, y) in the top half of the tile and (x, y + 8)).
// Each thread replays its pixels front to back exactly as the forward did
// (same float operations, so T and every accept / early-out decision match the
// forward bit-for-bit), carrying the residual colour C - T_final*bg - (front
// contributions) as the reference does, folded into one scalar (its dot
// product with the pixel's output gradient). Each warp visits only the staged
// splats that reach one of its two row bands (the forward's exact footprint
// test per band, kept from the forward as one byte per intersection; the list
// is built once per batch, raster_common.cuh), and skips the pixel step of a
// band the splat cannot reach; each lane forms its pixels' contribution to the
// splat's 10 gradient lanes, the warp sums them with a 10-value butterfly (12 shuffles),
// the sums are accumulated per splat in shared memory across the tile's 4
// warps, and each (splat, tile) leaves with three 16-byte vector atomics
// (red.global.add.v4.f32) into a 12-lane row.
// The alpha / T chain uses exact IEEE operations; the gradient arithmetic,
// which is tolerance-checked, uses fused multiply-adds and approximate
// reciprocal and square root, and sums the screen-space offsets weighted by
// d loss / d sigma so that the conic multiplies them once per (splat, tile).
// Colours are clamped once per splat while staging; the colour-gradient
// gates (raw colour >= 0) are per-splat constants applied once at the flush.
#include "raster_common.cuh"

namespace bsx {

namespace {

constexpr int kGradLanes = 10;  // xy(2) conic(3) rgb(3) alpha refine

struct BwdArgs {
    const uint32_t* isect_gid;
    const uint32_t* tile_offsets;
    const float* projected;
    const float* image;     // [H,W,4]
    const float* v_output;  // [H,W,4]
    float* v_grad;          // [N,12]
    const uint8_t* isect_mask;  // [M] band masks the forward computed for these ranges, or null: compute them
    const uint32_t* order;  // launch order of the tiles (block b replays tile order[b])
    uint32_t tbw, num_tiles, w, h;
    float bg_r, bg_g, bg_b;
};

// Pairwise butterfly step: lanes with `bit` clear keep value k and send k+h,
// lanes with it set keep k+h and send k; each keeps the pair sum.
template <int H, int N>
__device__ __forceinline__ void butterfly_step(float (&v)[N], bool up, int lane_xor) {
#pragma unroll
    for (int k = 0; k < H; ++k) {
        const float hi = k + H < N ? v[k + H] : 0.0f;
        const float send = up ? v[k] : hi;
        const float keep = up ? hi : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, lane_xor);
    }
}

// Sum 10 per-lane values over the warp with 12 shuffles (5 + 3 + 2 + 1 + 1).
// Returns on lane l the total of value warp_sum10_index(l) (both lanes of an
// even/odd pair hold it); lanes whose index is >= 10 hold padding.
__device__ __forceinline__ int warp_sum10_index(int lane) {
    const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1;
    const int w = 2 * b2 + b1;            // index within the 3 values of level 3
    const int u = 3 * b3 + w;             // index within the 5 values of level 2
    return (w < 3 && u < 5) ? 5 * b4 + u : 16;
}
__device__ __forceinline__ float warp_sum10(float (&v)[10], int lane) {
    butterfly_step<5, 10>(v, lane & 16, 16);
    float u[5] = {v[0], v[1], v[2], v[3], v[4]};
    butterfly_step<3, 5>(u, lane & 8, 8);
    float w[3] = {u[0], u[1], u[2]};
    butterfly_step<2, 3>(w, lane & 4, 4);
    float x[2] = {w[0], w[1]};
    butterfly_step<1, 2>(x, lane & 2, 2);
    return x[0] + __shfl_xor_sync(0xffffffffu, x[0], 1);
}

// Per-pixel replay state and constants.
//
// The colour residual is carried as one scalar. With s_c the residual colour
// C_c - T_final bg_c - (front contributions) of channel c and vo the pixel's
// output gradient, the reference's d loss / d alpha is
//   (sum_c (T cl_c - s_c) vo_c + (vo_a - bg.vo) T_final) / (1 - alpha)
// = (T (cl . vo) - E) / (1 - alpha),   E = s . vo - (vo_a - bg.vo) T_final,
// and each splat lowers E by vis (cl . vo). Initially
// E = C . vo - T_final vo_a (the background terms cancel).
struct PixelBwd {
    float T, E;                     // transmittance, scalar colour residual
    float vor, vog, vob;            // v_out rgb
    float inv_fa;                   // 1 / max(final alpha, 1e-5)
    float pcy;                      // pixel centre y
    bool done;
};

__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float sqrt_approx(float x) {
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void pixel_init(PixelBwd& P, const BwdArgs& a, uint32_t px, uint32_t py) {
    P.T = 1.0f;
    P.E = 0.0f;
    P.vor = P.vog = P.vob = 0.0f;
    P.inv_fa = 0.0f;
    P.pcy = (float)py + 0.5f;
    P.done = !(px < a.w && py < a.h);
    if (!P.done) {
        const size_t pid = (size_t)py * a.w + px;
        const float4 o = __ldg(reinterpret_cast<const float4*>(a.image) + pid);
        const float4 vo = __ldg(reinterpret_cast<const float4*>(a.v_output) + pid);
        P.vor = vo.x;
        P.vog = vo.y;
        P.vob = vo.z;
        P.E = __fmaf_rn(o.x, vo.x, __fmaf_rn(o.y, vo.y, __fmaf_rn(o.z, vo.z, -(1.0f - o.w) * vo.w)));
        P.inv_fa = __frcp_rn(bsx_max(o.w, 1.0e-5f));
    }
}

// One pixel's step of the replay for one splat: exact forward arithmetic for
// sigma / alpha / T, then the pixel's gradient contribution added into gv:
//   gv[0..1]  sum vsig (dx, dy)        (the conic is applied at the flush)
//   gv[2..4]  sum vsig (dx dx, dx dy, dy dy)   (halved at the flush)
//   gv[5..7]  sum vis vo_rgb,  gv[8] sum d loss / d opacity-alpha * gauss,
//   gv[9]     sum |(w, h) (conic (dx, dy) vsig)| / final alpha
// with (dx, dy) = pixel centre - splat mean.
template <bool SMOOTH, bool REFINE>
__device__ __forceinline__ bool pixel_step(PixelBwd& P, float dx0, float hxx, float xy, float sy, float hc11,
                                           float ca, float thr, float clr, float clg, float clb,
                                           const float4* rr, float (&gv)[10]) {
    if (P.done) return false;
    const float dyp = P.pcy - sy;
    const float sigma = bsx_sigma_row(hxx, xy, hc11, dyp);
    if (!(sigma >= 0.0f) || sigma > thr) return false;
    const float gauss = bsx_expf_raster(-sigma);
    const float cg = ca * gauss;
    const float alpha = bsx_min(0.999f, cg);
    const float wc = SMOOTH ? cutoff_weight(alpha) : (alpha >= 1.0f / 255.0f ? 1.0f : 0.0f);
    if (!(wc > 0.0f)) return false;
    const float ae = alpha * wc;
    const float one_m = 1.0f - ae;
    const float next_t = P.T * one_m;
    if (next_t <= 1.0e-4f) {
        P.done = true;
        return false;
    }
    // gradient arithmetic (tolerance-checked): fused operations allowed
    const float T = P.T;
    const float vis = ae * T;
    // colour lanes: gated on raw colour >= 0 at the flush
    gv[5] = __fmaf_rn(vis, P.vor, gv[5]);
    gv[6] = __fmaf_rn(vis, P.vog, gv[6]);
    gv[7] = __fmaf_rn(vis, P.vob, gv[7]);
    const float cv = __fmaf_rn(clr, P.vor, __fmaf_rn(clg, P.vog, clb * P.vob));
    const float vae = __fmaf_rn(T, cv, -P.E) * rcp_approx(one_m);
    const float valpha = SMOOTH ? vae * (wc + alpha * cutoff_weight_deriv(alpha)) : vae;
    if (cg <= 0.999f) {
        const float vsig = -alpha * valpha;
        const float a = vsig * dx0, b = vsig * dyp;
        gv[0] += a;
        gv[1] += b;
        gv[2] = __fmaf_rn(a, dx0, gv[2]);
        gv[3] = __fmaf_rn(a, dyp, gv[3]);
        gv[4] = __fmaf_rn(b, dyp, gv[4]);
        gv[8] = __fmaf_rn(valpha, gauss, gv[8]);
        if (REFINE) {
            // the splat's conic rows scaled by the image size: (c00 w, c01 w, c01 h, c11 h)
            const float4 r = *rr;
            const float ax = __fmaf_rn(r.x, a, r.y * b), ay = __fmaf_rn(r.z, a, r.w * b);
            gv[9] = __fmaf_rn(sqrt_approx(__fmaf_rn(ax, ax, ay * ay)), P.inv_fa, gv[9]);
        }
    }
    P.E = __fmaf_rn(-vis, cv, P.E);
    P.T = next_t;
    return true;
}

// Two pixels per thread (rows y and y + 8 of the tile), 128 threads per tile.
constexpr int kBwdPixThreads = 128;

// Bounded to 56 registers (nine resident blocks per SM; the refine variant
// spills 8 bytes): with the per-warp visit lists this measured 2 % faster than
// 64 registers at eight blocks (before the lists, nine blocks were 6 % slower).
template <bool SMOOTH, bool REFINE>
__global__ void __launch_bounds__(kBwdPixThreads, 9) raster_bwd_kernel(const BwdArgs a) {
    __shared__ float4 s_a[kBwdPixThreads];  // x, y, c00, c01
    __shared__ float4 s_b[kBwdPixThreads];  // c11, opacity, max(r,0), max(g,0)
    __shared__ float2 s_c[kBwdPixThreads];  // max(b,0), ln(255 o) + margin
    __shared__ float4 s_d[REFINE ? kBwdPixThreads : 1];  // refine rows (c00 w, c01 w, c01 h, c11 h)
    __shared__ uint32_t s_mask[kBwdPixThreads];  // bits 0-7 warp row bands, 8-10 colour gates
    __shared__ uint8_t s_list[kBwdPixThreads / 32][kBwdPixThreads];  // per warp: the staged splats it visits
    __shared__ uint32_t s_gid[kBwdPixThreads];
    __shared__ float s_grad[kBwdPixThreads][kGradLanes + 1];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sum_idx = warp_sum10_index(lane);
    const uint32_t tile = __ldg(a.order + blockIdx.x);
    const uint32_t lo = __ldg(a.tile_offsets + tile * 2), hi = __ldg(a.tile_offsets + tile * 2 + 1);
    if (hi <= lo) return;
    const uint32_t ox = (tile % a.tbw) * kTile, oy = (tile / a.tbw) * kTile;
    const uint32_t lx = compact_bits_16(threadIdx.x), ly = compact_bits_16(threadIdx.x >> 1);
    const uint32_t wshift = 2 * warp;  // this warp's two band bits in s_mask
    const uint32_t px = ox + lx;
    const float pcx = (float)px + 0.5f;
    const float margin = SMOOTH ? kMarginSmooth : kMarginHard;
    const float wf = (float)a.w, hf = (float)a.h;
    PixelBwd PA, PB;
    pixel_init(PA, a, px, oy + ly);
    pixel_init(PB, a, px, oy + ly + 8);

    for (uint32_t batch = lo; batch < hi; batch += kBwdPixThreads) {
        if (__syncthreads_count(PA.done && PB.done) == kBwdPixThreads) break;
        const uint32_t n = min((uint32_t)kBwdPixThreads, hi - batch);
        if (threadIdx.x < n) {
            const uint32_t g = __ldg(a.isect_gid + batch + threadIdx.x);
            const float4* row = reinterpret_cast<const float4*>(a.projected + (size_t)g * BSX_PROJECTED_LANES);
            const float4 ra = __ldg(row), rb = __ldg(row + 1), rc = __ldg(row + 2);
            s_a[threadIdx.x] = ra;
            s_b[threadIdx.x] = make_float4(rb.x, rb.y, bsx_max(rb.z, 0.0f), bsx_max(rb.w, 0.0f));
            s_c[threadIdx.x] = make_float2(bsx_max(rc.x, 0.0f), rc.z + margin);
            if (REFINE) s_d[threadIdx.x] = make_float4(ra.z * wf, ra.w * wf, ra.w * hf, rb.x * hf);
            const uint32_t gates = (rb.z >= 0.0f ? 256u : 0u) | (rb.w >= 0.0f ? 512u : 0u) | (rc.x >= 0.0f ? 1024u : 0u);
            // the forward's masks of these indices (same splat rows, tile, margin and
            // arithmetic), when it left them
            const uint32_t vm = a.isect_mask ? (uint32_t)__ldg(a.isect_mask + batch + threadIdx.x)
                                             : warp_visit_mask(ra.x, ra.y, ra.z, ra.w, rb.x, rc.z + margin, ox, oy);
            s_mask[threadIdx.x] = vm | gates;
            s_gid[threadIdx.x] = g;
#pragma unroll
            for (int k = 0; k <= kGradLanes; ++k) s_grad[threadIdx.x][k] = 0.0f;
        }
        __syncthreads();
        uint8_t* list = s_list[warp];
        const uint32_t nvis = warp_visit_list<kBwdPixThreads>(s_mask, n, wshift, list);
        for (uint32_t i = 0; i < nvis; ++i) {
            const uint32_t t = list[i];
            const uint32_t bands = (s_mask[t] >> wshift) & 3u;  // warp-uniform, non-zero
            const float4 A = s_a[t];
            const float4 B = s_b[t];
            const float2 Cc = s_c[t];
            const float4* rr = &s_d[REFINE ? t : 0];
            const float dx0 = pcx - A.x;
            const float hxx = bsx_sigma_hxx(A.z, dx0);
            const float xy = A.w * dx0;
            const float hc11 = 0.5f * B.x;
            float gv[kGradLanes];
#pragma unroll
            for (int k = 0; k < kGradLanes; ++k) gv[k] = 0.0f;
            // a band the splat cannot reach has every sigma > thr: its pixel step is a no-op
            bool contrib = (bands & 1u) && pixel_step<SMOOTH, REFINE>(PA, dx0, hxx, xy, A.y, hc11, B.y, Cc.y, B.z,
                                                                      B.w, Cc.x, rr, gv);
            if (bands & 2u)
                contrib |= pixel_step<SMOOTH, REFINE>(PB, dx0, hxx, xy, A.y, hc11, B.y, Cc.y, B.z, B.w, Cc.x, rr, gv);
            if (__any_sync(0xffffffffu, contrib)) {
                const float tot = warp_sum10(gv, lane);
                if (!(lane & 1) && sum_idx < kGradLanes) atomicAdd(&s_grad[t][sum_idx], tot);
            } else if (__all_sync(0xffffffffu, PA.done && PB.done)) {
                break;  // warp-uniform: a finished pixel never contributes, so this is tested only here
            }
        }
        __syncthreads();
        if (threadIdx.x < n) {
            const float* sgr = s_grad[threadIdx.x];
            const uint32_t gates = s_mask[threadIdx.x];
            const float vr = (gates & 256u) ? sgr[5] : 0.0f, vg = (gates & 512u) ? sgr[6] : 0.0f,
                        vb = (gates & 1024u) ? sgr[7] : 0.0f;
            bool any = false;
#pragma unroll
            for (int k = 0; k < kGradLanes; ++k) any = any || sgr[k] != 0.0f;
            if (any) {
                // d loss / d mean2d = -conic (sum vsig (dx, dy)) in the reference's
                // d = mean - pixel convention; the conic lanes take the halving
                const float4 A = s_a[threadIdx.x];
                const float c11 = s_b[threadIdx.x].x;
                const float gx = -__fmaf_rn(A.z, sgr[0], A.w * sgr[1]);
                const float gy = -__fmaf_rn(A.w, sgr[0], c11 * sgr[1]);
                float4* dst = reinterpret_cast<float4*>(a.v_grad + (size_t)s_gid[threadIdx.x] * kGradStride);
                atomicAdd(dst, make_float4(gx, gy, 0.5f * sgr[2], sgr[3]));
                atomicAdd(dst + 1, make_float4(0.5f * sgr[4], vr, vg, vb));
                atomicAdd(dst + 2, make_float4(sgr[8], sgr[9], 0.0f, 0.0f));
            }
        }
    }
}

}  // namespace

bsx_status launch_raster_bwd(bsx_ctx* ctx, const uint32_t* isect_gid, const uint32_t* tile_offsets,
                             const float* projected, const float* image, const float* v_output, float* v_grad,
                             const uint8_t* isect_mask, const uint32_t* order, const bsx_project_uniforms& u,
                             const float bg[3], int smooth, int refine) {
    BwdArgs a;
    a.isect_gid = isect_gid;
    a.tile_offsets = tile_offsets;
    a.projected = projected;
    a.image = image;
    a.v_output = v_output;
    a.v_grad = v_grad;
    a.isect_mask = isect_mask;
    a.tbw = u.tile_bw;
    a.num_tiles = u.tile_bw * u.tile_bh;
    a.w = u.img_w;
    a.h = u.img_h;
    a.bg_r = bg[0];
    a.bg_g = bg[1];
    a.bg_b = bg[2];
    const uint32_t blocks = a.num_tiles;
    // launch order: the forward's (heaviest tiles first) when given, else from
    // these ranges into the operator's own buffer (the forward's order stays intact)
    if (order) {
        a.order = order;
    } else {
        bsx_status s = ensure(ctx, ctx->ref_order, (size_t)blocks * 4);
        if (s == BSX_OK) s = tile_order(ctx, tile_offsets, blocks, ctx->ref_order.as<uint32_t>());
        if (s != BSX_OK) return s;
        a.order = ctx->ref_order.as<uint32_t>();
    }
    prof_begin(ctx);
    if (smooth) {
        if (refine) raster_bwd_kernel<true, true><<<blocks, kBwdPixThreads, 0, ctx->stream>>>(a);
        else raster_bwd_kernel<true, false><<<blocks, kBwdPixThreads, 0, ctx->stream>>>(a);
    } else {
        if (refine) raster_bwd_kernel<false, true><<<blocks, kBwdPixThreads, 0, ctx->stream>>>(a);
        else raster_bwd_kernel<false, false><<<blocks, kBwdPixThreads, 0, ctx->stream>>>(a);
    }
    return post_launch(ctx, "raster_bwd_kernel");
}

}  // namespace bsx
