// bounds.cu - percentile bounds of the splat means (the trainer's BoundingBox).
//
// Restates bounds_from_pos (crates/brush-train/src/splat_init.rs:130-158):
// per axis, keep the finite coordinates (n of them), take the order
// statistics lo = trunc(f32((1 - p) / 2) * f32(n)) and
// hi = min(n - 1, trunc(f32((1 + p) / 2) * f32(n))) under f32::total_cmp, and
// return center (max + min) / 2 and extent (max - min) / 2
// (BoundingBox::from_min_max, crates/brush-render/src/bounding_box.rs:8-13); an
// axis without a finite coordinate gives the box [-1, 1]^3.
//
// The order statistics come from this library's radix sort of order-preserving
// keys: a float with bits b maps to ~b when its sign bit is set and to
// b | 0x80000000 otherwise, which orders as total_cmp does (-0 before +0);
// non-finite coordinates map to 0xFFFFFFFF, after every finite key.
#include <cstring>

#include "common.cuh"

namespace bsx {

namespace {

constexpr int kBoundsThreads = 256;

__device__ __forceinline__ uint32_t total_order_key(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__global__ void __launch_bounds__(kBoundsThreads)
    bounds_keys_kernel(const float* __restrict__ means, uint32_t stride, uint32_t n, int axis,
                       uint32_t* __restrict__ keys, uint32_t* __restrict__ finite) {
    const uint32_t i = blockIdx.x * kBoundsThreads + threadIdx.x;
    bool ok = false;
    if (i < n) {
        const float x = __ldg(means + (size_t)i * stride + axis);
        ok = bsx_is_finite(x);
        keys[i] = ok ? total_order_key(x) : 0xFFFFFFFFu;
    }
    const uint32_t c = __popc(__ballot_sync(0xffffffffu, ok));
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(finite, c);
}

// out[0..1] = (lo value, hi value) of the sorted finite keys; out[2] = count as bits.
__global__ void bounds_pick_kernel(const uint32_t* __restrict__ sorted, const uint32_t* __restrict__ finite,
                                   float percentile, float* __restrict__ out) {
    const uint32_t n = *finite;
    float lo_v = 0.0f, hi_v = 0.0f;
    if (n > 0) {
        const float fn = (float)n;
        const uint32_t lo = (uint32_t)(((1.0f - percentile) / 2.0f) * fn);
        const uint32_t hi = min(n - 1, (uint32_t)(((1.0f + percentile) / 2.0f) * fn));
        lo_v = key_value(sorted[min(lo, n - 1)]);
        hi_v = key_value(sorted[hi]);
    }
    out[0] = lo_v;
    out[1] = hi_v;
    out[2] = __uint_as_float(n);
}

}  // namespace

}  // namespace bsx

using namespace bsx;

extern "C" bsx_status bsx_splat_bounds(bsx_ctx* ctx, const float* d_means, uint32_t stride, uint32_t n,
                                       float percentile, float center[3], float extent[3]) {
    if (!ctx || !center || !extent || (n && !d_means) || stride < 3) return BSX_ERR_INVALID_ARG;
    if (!(percentile >= 0.0f && percentile <= 1.0f)) return fail(ctx, BSX_ERR_INVALID_ARG, "percentile out of [0, 1]");
    cudaSetDevice(ctx->device);
    // keys, their sorted copy and the sort's value output (each 256-byte aligned),
    // then 3 counters and 9 result words
    const size_t nn = ((size_t)(n ? n : 1) + 63) / 64 * 64;
    bsx_status s = ensure(ctx, ctx->bounds_tmp, (3 * nn + 16) * 4);
    if (s != BSX_OK) return s;
    uint32_t* keys = ctx->bounds_tmp.as<uint32_t>();
    uint32_t* sorted = keys + nn;
    uint32_t* vals_out = sorted + nn;
    uint32_t* counters = keys + 3 * nn;  // [3]
    float* picks = reinterpret_cast<float*>(counters + 4);  // [3][3]
    s = check_cuda(ctx, cudaMemsetAsync(counters, 0, 16 * 4, ctx->stream), "memset bounds counters");
    if (s != BSX_OK) return s;
    for (int axis = 0; axis < 3 && n; ++axis) {
        prof_begin(ctx);
        bounds_keys_kernel<<<(n + kBoundsThreads - 1) / kBoundsThreads, kBoundsThreads, 0, ctx->stream>>>(
            d_means, stride, n, axis, keys, counters + axis);
        if ((s = post_launch(ctx, "bounds_keys_kernel")) != BSX_OK) return s;
        // the keys double as the (unused) values of the pair sort
        if ((s = radix_sort_pairs(ctx, keys, keys, n, 32, sorted, vals_out)) != BSX_OK) return s;
        prof_begin(ctx);
        bounds_pick_kernel<<<1, 1, 0, ctx->stream>>>(sorted, counters + axis, percentile, picks + 3 * axis);
        if ((s = post_launch(ctx, "bounds_pick_kernel")) != BSX_OK) return s;
    }
    float h[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    if (n) {
        s = check_cuda(ctx, cudaMemcpyAsync(h, picks, sizeof h, cudaMemcpyDeviceToHost, ctx->stream), "bounds readback");
        if (s == BSX_OK) s = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "bounds synchronise");
        if (s != BSX_OK) return s;
    }
    bool empty = n == 0;
    for (int a = 0; a < 3; ++a) {
        uint32_t c;
        std::memcpy(&c, h + 3 * a + 2, 4);
        empty = empty || c == 0;
    }
    for (int a = 0; a < 3; ++a) {
        const float mn = empty ? -1.0f : h[3 * a], mx = empty ? 1.0f : h[3 * a + 1];
        center[a] = (mx + mn) / 2.0f;
        extent[a] = (mx - mn) / 2.0f;
    }
    return BSX_OK;
}
