// raster_bwd.cu - tile rasterizer, backward.
//
// Restates rasterize_backwards_kernel
// (crates/brush-render-bwd/src/kernels/rasterize_backwards.rs:79-443). One
// warp per tile; each lane owns one splat of the current 32-splat batch and
// accumulates that splat's 11 gradient lanes in registers. Per-pixel state
// (residual colour C - sum(front contributions) - T_final*bg, and
// transmittance T) lives in shared memory and is replayed front to back on a
// diagonal wavefront: at step i lane l handles pixel i-l, so every pixel sees
// the splats in depth order. The replay performs exactly the forward pass's
// float operations, so T and every accept / early-out decision match the
// forward bit-for-bit. Gradients leave registers once per (splat, tile) as
// three 16-byte vector atomics (red.global.add.v4.f32) into a 12-lane row.
#include "splat_math.cuh"

namespace bsx {

namespace {

constexpr int kBwdWarps = 4;  // tiles per block
constexpr int kBwdThreads = kBwdWarps * 32;
constexpr float kMarginHard = 1.0e-3f;
constexpr float kMarginSmooth = 0.25f;

__device__ __forceinline__ float cutoff_weight(float a) {
    const float mid = 1.0f / 255.0f, band = 1.0e-3f;
    float t = bsx_clamp((a - (mid - 0.5f * band)) / band, 0.0f, 1.0f);
    return t * t * (3.0f - 2.0f * t);
}
__device__ __forceinline__ float cutoff_weight_deriv(float a) {
    const float mid = 1.0f / 255.0f, band = 1.0e-3f;
    const float lo = mid - 0.5f * band, hi = mid + 0.5f * band;
    const bool inside = a > lo && a < hi;
    const float t = (a - lo) / band;
    return inside ? (6.0f * t - 6.0f * t * t) / band : 0.0f;
}

struct BwdArgs {
    const uint32_t* isect_gid;
    const uint32_t* tile_offsets;
    const float* projected;
    const float* image;     // [H,W,4]
    const float* v_output;  // [H,W,4]
    float* v_grad;          // [N,12]
    uint32_t tbw, num_tiles, w, h;
    float bg_r, bg_g, bg_b;
};

template <bool SMOOTH, bool REFINE>
__global__ void __launch_bounds__(kBwdThreads) raster_bwd_kernel(const BwdArgs a) {
    __shared__ float4 s_state[kBwdWarps][kTilePixels];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t tile = blockIdx.x * kBwdWarps + warp;
    if (tile >= a.num_tiles) return;
    const uint32_t lo = __ldg(a.tile_offsets + tile * 2), hi = __ldg(a.tile_offsets + tile * 2 + 1);
    if (hi <= lo) return;
    const uint32_t ox = (tile % a.tbw) * kTile, oy = (tile / a.tbw) * kTile;
    float4* st = s_state[warp];
    const float4* img4 = reinterpret_cast<const float4*>(a.image);
    const float4* vo4 = reinterpret_cast<const float4*>(a.v_output);
    for (int p = lane; p < kTilePixels; p += 32) {
        const uint32_t px = ox + (p % kTile), py = oy + (p / kTile);
        float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (px < a.w && py < a.h) {
            const float4 o = __ldg(img4 + (size_t)py * a.w + px);
            const float tf = 1.0f - o.w;
            s = make_float4(o.x - tf * a.bg_r, o.y - tf * a.bg_g, o.z - tf * a.bg_b, 1.0f);
        }
        st[p] = s;
    }
    __syncwarp();
    const float margin = SMOOTH ? kMarginSmooth : kMarginHard;
    const float wf = (float)a.w, hf = (float)a.h;
    const uint32_t count = hi - lo;
    for (uint32_t b0 = 0; b0 < count; b0 += 32) {
        const uint32_t nb = min(32u, count - b0);
        const bool active = (uint32_t)lane < nb;
        uint32_t g = 0;
        float4 A = make_float4(0, 0, 0, 0), B = A, C = A;
        if (active) {
            g = __ldg(a.isect_gid + lo + b0 + lane);
            const float4* row = reinterpret_cast<const float4*>(a.projected + (size_t)g * BSX_PROJECTED_LANES);
            A = __ldg(row);
            B = __ldg(row + 1);
            C = __ldg(row + 2);
        }
        const float sx = A.x, sy = A.y, c00 = A.z, c01 = A.w, c11 = B.x, ca = B.y;
        const float craw = B.z, cgraw = B.w, cbraw = C.x, pt = C.z;
        const float clr = bsx_max(craw, 0.0f), clg = bsx_max(cgraw, 0.0f), clb = bsx_max(cbraw, 0.0f);
        float g_xy_x = 0, g_xy_y = 0, g_c0 = 0, g_c1 = 0, g_c2 = 0, g_r = 0, g_g = 0, g_b = 0, g_a = 0, g_ref = 0;
        const uint32_t steps = nb + kTilePixels - 1;
        for (uint32_t i = 0; i < steps; ++i) {
            const int p = (int)i - lane;
            if (active && p >= 0 && p < kTilePixels) {
                float4 s = st[p];
                if (s.w > 1.0e-4f) {
                    const uint32_t px = ox + (p % kTile), py = oy + (p / kTile);
                    const float dx = sx - ((float)px + 0.5f);
                    const float dy = sy - ((float)py + 0.5f);
                    const float sigma = 0.5f * (c00 * dx * dx + c11 * dy * dy) + c01 * dx * dy;
                    if (sigma <= pt + margin) {
                        const float gauss = bsx_expf(-sigma);
                        const float alpha = bsx_min(0.999f, ca * gauss);
                        const float wc = SMOOTH ? cutoff_weight(alpha) : (alpha >= 1.0f / 255.0f ? 1.0f : 0.0f);
                        if (sigma >= 0.0f && wc > 0.0f) {
                            const float ae = alpha * wc;
                            const float next_t = s.w * (1.0f - ae);
                            if (next_t <= 1.0e-4f) {
                                st[p].w = 0.0f;
                            } else {
                                const float vis = ae * s.w;
                                const size_t pid = (size_t)py * a.w + px;
                                const float4 vo = __ldg(vo4 + pid);
                                const float fa = __ldg(a.image + pid * 4 + 3);
                                const float tf = 1.0f - fa;
                                const float vow = (vo.w - (a.bg_r * vo.x + a.bg_g * vo.y + a.bg_b * vo.z)) * tf;
                                g_r += craw >= 0.0f ? vis * vo.x : 0.0f;
                                g_g += cgraw >= 0.0f ? vis * vo.y : 0.0f;
                                g_b += cbraw >= 0.0f ? vis * vo.z : 0.0f;
                                const float ra = 1.0f / (1.0f - ae);
                                const float dot_rgb = ((s.w * clr - s.x) * vo.x + (s.w * clg - s.y) * vo.y +
                                                       (s.w * clb - s.z) * vo.z) * ra;
                                const float nrx = s.x - vis * clr, nry = s.y - vis * clg, nrz = s.z - vis * clb;
                                const float vae = dot_rgb + vow * ra;
                                const float dw = SMOOTH ? cutoff_weight_deriv(alpha) : 0.0f * alpha;
                                const float valpha = vae * (wc + alpha * dw);
                                const float vsig = -alpha * valpha;
                                const float vxx = vsig * (c00 * dx + c01 * dy);
                                const float vxy = vsig * (c01 * dx + c11 * dy);
                                if (ca * gauss <= 0.999f) {
                                    g_c0 += 0.5f * vsig * dx * dx;
                                    g_c1 += vsig * dx * dy;
                                    g_c2 += 0.5f * vsig * dy * dy;
                                    g_xy_x += vxx;
                                    g_xy_y += vxy;
                                    g_a += valpha * gauss;
                                    if (REFINE) {
                                        const float len = sqrtf(vxx * wf * vxx * wf + vxy * hf * vxy * hf);
                                        g_ref += len / bsx_max(fa, 1.0e-5f);
                                    }
                                }
                                st[p] = make_float4(nrx, nry, nrz, next_t);
                            }
                        }
                    }
                }
            }
            __syncwarp();
        }
        if (active) {
            float4* dst = reinterpret_cast<float4*>(a.v_grad + (size_t)g * kGradStride);
            atomicAdd(dst, make_float4(g_xy_x, g_xy_y, g_c0, g_c1));
            atomicAdd(dst + 1, make_float4(g_c2, g_r, g_g, g_b));
            atomicAdd(dst + 2, make_float4(g_a, g_ref, 0.0f, 0.0f));
        }
    }
}

}  // namespace

bsx_status launch_raster_bwd(bsx_ctx* ctx, const uint32_t* isect_gid, const uint32_t* tile_offsets,
                             const float* projected, const float* image, const float* v_output, float* v_grad,
                             const bsx_project_uniforms& u, const float bg[3], int smooth, int refine) {
    BwdArgs a;
    a.isect_gid = isect_gid;
    a.tile_offsets = tile_offsets;
    a.projected = projected;
    a.image = image;
    a.v_output = v_output;
    a.v_grad = v_grad;
    a.tbw = u.tile_bw;
    a.num_tiles = u.tile_bw * u.tile_bh;
    a.w = u.img_w;
    a.h = u.img_h;
    a.bg_r = bg[0];
    a.bg_g = bg[1];
    a.bg_b = bg[2];
    const uint32_t blocks = (a.num_tiles + kBwdWarps - 1) / kBwdWarps;
    prof_begin(ctx);
    if (smooth) {
        if (refine) raster_bwd_kernel<true, true><<<blocks, kBwdThreads, 0, ctx->stream>>>(a);
        else raster_bwd_kernel<true, false><<<blocks, kBwdThreads, 0, ctx->stream>>>(a);
    } else {
        if (refine) raster_bwd_kernel<false, true><<<blocks, kBwdThreads, 0, ctx->stream>>>(a);
        else raster_bwd_kernel<false, false><<<blocks, kBwdThreads, 0, ctx->stream>>>(a);
    }
    return post_launch(ctx, "raster_bwd_kernel");
}

}  // namespace bsx
