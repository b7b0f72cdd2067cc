// tile_walk.cuh - warp-cooperative walk over the tile boxes of 32 splats.
//
// The projection counts, and the emission writes, every tile of a splat's
// tile box that passes the StopThePop test (tile_contrib). One thread per
// splat walking its own box leaves most lanes idle: a warp runs as long as
// its largest box (on the benchmark scenes a lane does useful work 13-28 % of
// the time). Here the warp's boxes are laid end to end, each box in row-major
// order (the reference's order, map_gaussians.rs:56-85), and the warp takes 32
// consecutive (splat, tile) candidates per iteration: a lane finds the splat
// owning candidate j by a binary search over the exclusive prefix of box
// areas, fetches that splat's box and conic from the owner lane by shuffles,
// and evaluates the same tile_contrib on the same floats. Decisions are
// therefore bit-identical to the per-thread loop, and hits of one splat come
// out in the same order.
#pragma once
#include "splat_math.cuh"

namespace bsx {

constexpr uint32_t kFullMask = 0xffffffffu;

// One lane's splat as seen by the walk; area 0 takes no part.
struct WalkSplat {
    uint32_t x0, y0, w, area;  // tile box origin, width, width * height
    float mx, my;              // projected mean
    S2 conic;
    float pt;                  // ln(255 * opacity)
};

// Per iteration of the walk, what a lane sees.
struct WalkStep {
    bool hit;        // candidate of this lane passes tile_contrib
    uint32_t owner;  // lane whose splat owns this lane's candidate
    uint32_t tx, ty; // the candidate tile
    uint32_t ballot; // hits of the whole warp this iteration
    uint32_t before; // hits of the owner's splat on lower lanes this iteration
    uint32_t own;    // hits of THIS lane's splat this iteration
};

__device__ __forceinline__ uint32_t lanes_below(uint32_t n) { return n >= 32 ? kFullMask : ((1u << n) - 1u); }

// Runs fn(step) once per iteration on every lane of the warp (all 32 lanes
// must call it with the same control flow).
template <typename Fn>
__device__ __forceinline__ void warp_tile_walk(const WalkSplat& me, Fn&& fn) {
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t incl = me.area;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t v = __shfl_up_sync(kFullMask, incl, d);
        if (lane >= (uint32_t)d) incl += v;
    }
    const uint32_t excl = incl - me.area;
    const uint32_t total = __shfl_sync(kFullMask, incl, 31);
    const float inv_w = me.area ? 1.0f / (float)me.w : 0.0f;
    for (uint32_t base = 0; base < total; base += 32) {
        const uint32_t j = base + lane;
        // largest lane whose exclusive prefix is <= j (empty boxes before the
        // owner have smaller prefixes, empty boxes after it larger ones)
        uint32_t o = 0;
#pragma unroll
        for (uint32_t step = 16; step; step >>= 1) {
            const uint32_t e = __shfl_sync(kFullMask, excl, o + step);
            if (e <= j) o += step;
        }
        const uint32_t oe = __shfl_sync(kFullMask, excl, o);
        const uint32_t ox0 = __shfl_sync(kFullMask, me.x0, o), oy0 = __shfl_sync(kFullMask, me.y0, o);
        const uint32_t ow = __shfl_sync(kFullMask, me.w, o);
        const float oinv = __shfl_sync(kFullMask, inv_w, o);
        const float mx = __shfl_sync(kFullMask, me.mx, o), my = __shfl_sync(kFullMask, me.my, o);
        const S2 c{__shfl_sync(kFullMask, me.conic.c00, o), __shfl_sync(kFullMask, me.conic.c01, o),
                   __shfl_sync(kFullMask, me.conic.c11, o)};
        const float opt = __shfl_sync(kFullMask, me.pt, o);
        WalkStep s;
        s.owner = o;
        s.hit = false;
        s.tx = s.ty = 0;
        if (j < total) {
            const uint32_t k = j - oe;
            // row = floor(k / w): (k + 0.5) / w lies at least 0.5/w inside the
            // bracket, far more than the float error; one correction step guards it
            uint32_t q = (uint32_t)(((float)k + 0.5f) * oinv);
            int32_t r = (int32_t)(k - q * ow);
            if (r < 0) {
                --q;
                r += (int32_t)ow;
            } else if (r >= (int32_t)ow) {
                ++q;
                r -= (int32_t)ow;
            }
            s.tx = ox0 + (uint32_t)r;
            s.ty = oy0 + q;
            s.hit = tile_contrib(s.tx, s.ty, mx, my, c, opt);
        }
        s.ballot = __ballot_sync(kFullMask, s.hit);
        const uint32_t ostart = oe > base ? oe - base : 0u;  // owner's first lane this iteration
        s.before = __popc(s.ballot & lanes_below(lane) & ~lanes_below(ostart));
        const uint32_t mstart = excl > base ? excl - base : 0u;
        const uint32_t mend = incl > base ? min(incl - base, 32u) : 0u;
        s.own = mstart < mend ? __popc(s.ballot & lanes_below(mend) & ~lanes_below(mstart)) : 0u;
        fn(s);
    }
}

}  // namespace bsx
