// raster_common.cuh - helpers shared by the forward and backward tile
// rasterizers: the pixel layout of a tile block, the smooth alpha cutoff and
// the per-warp footprint test used to skip splats a warp cannot see.
//
// Pixel layout (both rasterizers): 128 threads per 16x16 tile, two pixels per
// thread. Thread t takes the reference's Morton position (x, y) of index t
// (crates/brush-render/src/kernels/helpers.rs:54-81; y < 8 since t < 128) and
// also owns (x, y + 8). Warp w therefore covers columns 8*(w>>1) .. +7 and the
// two row bands 4*(w&1) .. +3 and 4*(w&1)+8 .. +11.
#pragma once
#include "splat_math.cuh"

namespace bsx {

// Rejection margin on sigma for the exponential-free pre-filter. With the
// hard cutoff the exact test is sigma <= ln(255 o) up to a few ulp of the
// shared exp/ln; the smooth ramp starts at alpha = 1/255 - 5e-4, i.e.
// ln(255 o) + 0.137.
constexpr float kMarginHard = 1.0e-3f;
constexpr float kMarginSmooth = 0.25f;

__device__ __forceinline__ uint32_t compact_bits_16(uint32_t v) {
    uint32_t x = v & 0x55555555u;
    x = (x | (x >> 1)) & 0x33333333u;
    x = (x | (x >> 2)) & 0x0F0F0F0Fu;
    x = (x | (x >> 4)) & 0x00FF00FFu;
    x = (x | (x >> 8)) & 0x0000FFFFu;
    return x;
}

// C^1 smoothstep ramp of width 1e-3 around alpha = 1/255 (the reference's
// smooth cutoff for finite-difference tests, rasterize.rs / rasterize_backwards.rs).
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

// Minimum over the rectangle [ax,bx] x [ay,by] (offsets d = pixel - mean) of
// q(d) = 0.5 (c00 dx^2 + c11 dy^2) + c01 dx dy for a positive-definite conic.
// If the origin lies outside the rectangle in x, the minimum lies on the
// x-edge facing it (the sub-level set is convex and contains the origin, so
// the segment from the origin to any boundary minimiser crosses that edge);
// likewise in y. q1 minimises along the x-edge through dxc, q2 along the
// y-edge through dyc; each 1-D minimiser is the clamped vertex of a convex
// parabola. When the origin lies inside the x-range, q1 is the value at a
// point of the rectangle and q2 the exact minimum (or 0), so min(q1, q2) is
// the minimum in every case. r01 = c01/c11, s01 = c01/c00.
__device__ __forceinline__ float rect_min_sigma(float ax, float bx, float ay, float by, float c00, float c01,
                                                float c11, float r01, float s01) {
    const float dxc = fminf(fmaxf(0.0f, ax), bx);
    const float dyc = fminf(fmaxf(0.0f, ay), by);
    const float dy1 = fminf(fmaxf(-r01 * dxc, ay), by);
    const float dx2 = fminf(fmaxf(-s01 * dyc, ax), bx);
    const float q1 = __fmaf_rn(0.5f * c00 * dxc, dxc, __fmaf_rn(0.5f * c11 * dy1, dy1, c01 * dxc * dy1));
    const float q2 = __fmaf_rn(0.5f * c00 * dx2, dx2, __fmaf_rn(0.5f * c11 * dyc, dyc, c01 * dx2 * dyc));
    return fminf(q1, q2);
}

// Bit 2w + b set: row band b of warp w of the tile block at (ox, oy) (band 0
// holds the warp's first pixels, band 1 its pixels 8 rows lower) has a pixel
// centre whose sigma can be <= thr. The test is the exact minimum of sigma over
// each of the warp's two 8x4 pixel-centre rectangles, less a rounding allowance of 1e-5 of
// the largest term magnitude over the tile (the float evaluation of sigma at a
// pixel and of the rectangle minimum each err by well under 1e-6 of it), so a
// cleared bit means no pixel of that warp passes the per-pixel pre-filter
// sigma <= thr. Non-positive-definite conics and non-finite values keep every
// warp (conservative).
__device__ __forceinline__ uint32_t warp_visit_mask(float sx, float sy, float c00, float c01, float c11, float thr,
                                                    uint32_t ox, uint32_t oy) {
    const float det = c00 * c11 - c01 * c01;
    if (!(c00 > 0.0f && c11 > 0.0f && det > 0.0f)) return 0xffu;
    const float r01 = __fdividef(c01, c11), s01 = __fdividef(c01, c00);
    const float x0 = (float)ox + 0.5f - sx, y0 = (float)oy + 0.5f - sy;
    const float dxm = fmaxf(fabsf(x0), fabsf(x0 + 15.0f)), dym = fmaxf(fabsf(y0), fabsf(y0 + 15.0f));
    const float smax = 0.5f * (c00 * dxm * dxm + c11 * dym * dym) + fabsf(c01) * dxm * dym;
    const float bound = thr + 1.0e-5f * (smax + 1.0f);
    uint32_t mask = 0u;
#pragma unroll 1
    for (int w = 0; w < 4; ++w) {
        const float ax = x0 + (float)(8 * (w >> 1)), bx = ax + 7.0f;
#pragma unroll
        for (int band = 0; band < 2; ++band) {
            const float ay = y0 + (float)(4 * (w & 1) + 8 * band), by = ay + 3.0f;
            const float q = rect_min_sigma(ax, bx, ay, by, c00, c01, c11, r01, s01);
            // NaN compares false: the band is kept
            if (!(q > bound)) mask |= 1u << (2 * w + band);
        }
    }
    return mask;
}

// The staged splats of a batch (indices t < n) that reach one of this warp's
// two row bands (its two bits at `wshift` in s_mask), in staging order: written
// to `list`, their count returned (warp-uniform). The warp then visits only
// these, instead of testing every staged splat's bits in its visit loop.
template <int kBatch>
__device__ __forceinline__ uint32_t warp_visit_list(const uint32_t* s_mask, uint32_t n, uint32_t wshift,
                                                    uint8_t* list) {
    static_assert(kBatch <= 256, "8-bit list entries");
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t below = (1u << lane) - 1u;
    uint32_t cnt = 0;
#pragma unroll
    for (uint32_t c = 0; c < (uint32_t)kBatch; c += 32) {
        if (c >= n) break;  // warp-uniform
        const uint32_t t = c + lane;
        const bool hit = t < n && ((s_mask[t] >> wshift) & 3u) != 0u;
        const uint32_t bal = __ballot_sync(0xffffffffu, hit);
        if (hit) list[cnt + __popc(bal & below)] = (uint8_t)t;
        cnt += __popc(bal);
    }
    __syncwarp();
    return cnt;
}

}  // namespace bsx
