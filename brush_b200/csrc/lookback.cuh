// lookback.cuh - decoupled look-back helpers shared by the scan and the
// projection pass's stream compaction (Merrill & Garland 2016).
#pragma once
#include "common.cuh"

namespace bsx {

constexpr uint64_t kFlagAgg = 1ull << 32;
constexpr uint64_t kFlagIncl = 2ull << 32;

// Look back from `tile` over predecessors' status words; called by warp 0.
// Returns the exclusive prefix of `tile` (valid on all lanes of warp 0).
__device__ __forceinline__ uint32_t lookback_exclusive(uint64_t* status, uint32_t tile, int* err) {
    const int lane = threadIdx.x & 31;
    uint32_t exclusive = 0;
    int64_t pred = (int64_t)tile - 1;
    uint32_t spins = 0;
    while (pred >= 0) {
        int64_t idx = pred - lane;
        uint64_t s = idx >= 0 ? ld_relaxed_u64(status + idx) : kFlagIncl;
        uint32_t flag = (uint32_t)(s >> 32);
        if (__any_sync(0xffffffffu, flag == 0)) {
            if (++spins > kSpinLimit) {
                set_error(err, kDevLookbackTimeout);
                break;
            }
            __nanosleep(64);
            continue;
        }
        uint32_t incl_mask = __ballot_sync(0xffffffffu, flag == 2);
        int first = incl_mask ? __ffs(incl_mask) - 1 : 32;
        uint32_t v = lane <= first ? (uint32_t)s : 0u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        exclusive += v;
        if (incl_mask) break;
        pred -= 32;
    }
    return exclusive;
}


// Publish a tile's aggregate, look back, publish its inclusive prefix.
// Must be called by all 32 lanes of warp 0. Returns the exclusive prefix.
__device__ __forceinline__ uint32_t lookback_publish(uint64_t* status, uint32_t tile, uint32_t aggregate, int* err) {
    uint32_t prefix = 0;
    if (tile == 0) {
        if ((threadIdx.x & 31) == 0) st_relaxed_u64(status, kFlagIncl | aggregate);
    } else {
        if ((threadIdx.x & 31) == 0) st_relaxed_u64(status + tile, kFlagAgg | aggregate);
        prefix = lookback_exclusive(status, tile, err);
        if ((threadIdx.x & 31) == 0) st_relaxed_u64(status + tile, kFlagIncl | (uint32_t)(prefix + aggregate));
    }
    return prefix;
}

}  // namespace bsx
