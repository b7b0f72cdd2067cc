// loss.cu - fused SSIM (11x11 Gaussian window, sigma 1.5) + L1 image loss.
//
// Restates image_loss_forward_kernel / image_loss_backward_kernel /
// image_l1_*_kernel (crates/brush-loss/src/lib.rs:232-890): per 16x16 tile and
// channel, the image and effective ground truth (packed RGBA8, optional
// background compositing and alpha mask) are staged with a halo in shared
// memory, the five moments (x, x^2, y, y^2, xy) are blurred separably, SSIM
// and its partials (d/d mu_x, d/d sigma_x^2, d/d sigma_xy; zero where SSIM is
// clamped) are formed, and for the backward the chain-weighted partials are
// blurred again. Summation order matches the reference (taps d = 1..5 as
// (left + right) * w[5-d], then the centre tap).
//
// The training form (loss_ssim_kernel, loss_grad_kernel; loss_l1_fused_kernel
// when the SSIM weight is 0) reads the rasterizer's [H,W,4] image directly,
// uses the constant chain 1/(3HW) of a mean reduction, writes the gradient
// straight into the [H,W,4] v_output layout the raster backward consumes
// (alpha lane 0), and emits per-block loss sums that a tiny kernel reduces in
// a fixed order. This removes the reference's permute/contiguous copies, the
// separate mean kernel and the zero-fill of the gradient image. Its blur taps
// accumulate by fused multiply-adds (same tap order; the loss map and gradient
// are checked against the CPU restatement to 1e-5 relative, not bit for bit),
// and this file is the one the build compiles with multiply-add contraction:
// nothing here is a discrete decision another stage must reproduce.
#include "common.cuh"

namespace bsx {

namespace {

constexpr int kBlock = 16;
constexpr int kHalo = 5;
constexpr int kShared = kBlock + 2 * kHalo;    // 26
constexpr int kExtended = kBlock + 4 * kHalo;  // 36
constexpr float kC1 = 0.01f * 0.01f;
constexpr float kC2 = 0.03f * 0.03f;
constexpr float kInv255 = 1.0f / 255.0f;

struct LossTaps { float w[11]; };

struct LossArgs {
    const float* pred;       // [C,H,W] or [H,W,4]
    const uint32_t* gt;      // [H,W]
    const float* dl_dmap;    // [C,H,W] (null: constant chain)
    float chain_const;
    float* out;              // map or gradient, [C,H,W] or [H,W,4]
    float* block_loss;       // per-block loss sums (fused form)
    uint32_t w, h;
    float l1_w, ssim_w;
    int composite, mask;
    float bg[3];
    LossTaps taps;
};

template <bool HWC4>
__device__ __forceinline__ float read_pred(const LossArgs& a, int c, uint32_t y, uint32_t x) {
    return HWC4 ? __ldg(a.pred + ((size_t)y * a.w + x) * 4 + c) : __ldg(a.pred + ((size_t)c * a.h + y) * a.w + x);
}

__device__ __forceinline__ void read_gt(const LossArgs& a, int c, uint32_t y, uint32_t x, float* gc, float* ga) {
    const uint32_t v = __ldg(a.gt + (size_t)y * a.w + x);
    *gc = (float)((v >> (c * 8u)) & 0xffu) * kInv255;
    *ga = (float)((v >> 24u) & 0xffu) * kInv255;
}

__device__ __forceinline__ float gt_eff(const LossArgs& a, int c, uint32_t y, uint32_t x, float* ga) {
    float gc;
    read_gt(a, c, y, x, &gc, ga);
    if (a.composite) gc = gc + (1.0f - *ga) * a.bg[c];
    return gc;
}

struct Ssim { float val, dmu1, dsig1, dsig12; };
// SSIM and its partials (lib.rs:193-209, :480-500). Reciprocals are fast
// (2 ulp); the loss is checked against the host restatement by tolerance.
__device__ __forceinline__ Ssim ssim_terms(float o0, float o1, float o2, float o3, float o4) {
    const float mu1 = o0, mu2 = o2;
    const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2;
    const float s1 = bsx_max(0.0f, o1 - mu1_sq);
    const float s2 = bsx_max(0.0f, o3 - mu2_sq);
    const float s12 = o4 - mu1 * mu2;
    const float a = mu1_sq + mu2_sq + kC1;
    const float b = s1 + s2 + kC2;
    const float ct = 2.0f * mu1 * mu2 + kC1;
    const float dt = 2.0f * s12 + kC2;
    const float inv_a = __fdividef(1.0f, a), inv_b = __fdividef(1.0f, b);
    const float inv_ab = inv_a * inv_b;
    const float cd = ct * dt * inv_ab;
    Ssim r;
    r.val = bsx_clamp(cd, -1.0f, 1.0f);
    const bool clamped = cd < -1.0f || cd > 1.0f;
    r.dmu1 = clamped ? 0.0f : 2.0f * mu2 * inv_ab * (dt - ct) - 2.0f * mu1 * cd * (inv_a - inv_b);
    r.dsig1 = clamped ? 0.0f : -cd * inv_b;
    r.dsig12 = clamped ? 0.0f : 2.0f * ct * inv_ab;
    return r;
}

// Stage pred and effective gt of an (ext x ext) region starting `halo` pixels
// before the tile into sx / sy (planar); out-of-image samples are zero.
template <bool HWC4>
__device__ __forceinline__ void stage_tile(const LossArgs& a, int c, int tile_x0, int tile_y0, int ext, int halo,
                                           float* sx, float* sy) {
    for (int tid = threadIdx.x; tid < ext * ext; tid += blockDim.x) {
        const int ly = tid / ext, lx = tid - ly * ext;
        const int gy = tile_y0 + ly - halo, gx = tile_x0 + lx - halo;
        float pv = 0.0f, ge = 0.0f;
        if (gy >= 0 && gx >= 0 && gy < (int)a.h && gx < (int)a.w) {
            pv = read_pred<HWC4>(a, c, gy, gx);
            float ga;
            ge = gt_eff(a, c, gy, gx, &ga);
        }
        sx[tid] = pv;
        sy[tid] = ge;
    }
}

// Horizontal moment blur: rows [0,rows) of the staged region (row stride
// ext), output columns [0,cols) centred at staged column col + 5; output is
// five planes of rows*cols.
__device__ __forceinline__ void hblur_moments(const float* X, const float* Y, int ext, int rows, int cols,
                                              const float* w, float* o) {
    const int plane = rows * cols;
    for (int tid = threadIdx.x; tid < plane; tid += blockDim.x) {
        const int ry = tid / cols, cx = tid - ry * cols;
        const int center = ry * ext + cx + kHalo;
        float sx = 0.f, sx2 = 0.f, sy = 0.f, sy2 = 0.f, sxy = 0.f;
#pragma unroll
        for (int d = 1; d < 6; ++d) {
            const float wd = w[5 - d];
            const float xl = X[center - d], yl = Y[center - d], xr = X[center + d], yr = Y[center + d];
            sx += (xl + xr) * wd;
            sx2 += (xl * xl + xr * xr) * wd;
            sy += (yl + yr) * wd;
            sy2 += (yl * yl + yr * yr) * wd;
            sxy += (xl * yl + xr * yr) * wd;
        }
        const float xc = X[center], yc = Y[center], wc = w[5];
        sx += xc * wc;
        sx2 += xc * xc * wc;
        sy += yc * wc;
        sy2 += yc * yc * wc;
        sxy += xc * yc * wc;
        o[tid] = sx;
        o[plane + tid] = sx2;
        o[2 * plane + tid] = sy;
        o[3 * plane + tid] = sy2;
        o[4 * plane + tid] = sxy;
    }
}

// Vertical blur of the five moment planes at (center_row, col).
__device__ __forceinline__ void vblur5(const float* hb, int plane, int cols, int center_row, int col, const float* w,
                                       float o[5]) {
#pragma unroll
    for (int k = 0; k < 5; ++k) o[k] = 0.0f;
#pragma unroll
    for (int d = 1; d < 6; ++d) {
        const float wd = w[5 - d];
        const int it = (center_row - d) * cols + col, ib = (center_row + d) * cols + col;
#pragma unroll
        for (int k = 0; k < 5; ++k) o[k] += (hb[k * plane + it] + hb[k * plane + ib]) * wd;
    }
    const int ic = center_row * cols + col;
#pragma unroll
    for (int k = 0; k < 5; ++k) o[k] += hb[k * plane + ic] * w[5];
}

// Forward loss map, reference layout [C,H,W]; grid (tx, ty, C).
template <bool HWC4>
__global__ void __launch_bounds__(256) loss_fwd_kernel(const __grid_constant__ LossArgs a) {
    __shared__ float s_x[kShared * kShared];
    __shared__ float s_y[kShared * kShared];
    __shared__ float s_h[5 * kShared * kBlock];
    __shared__ float w[11];
    if (threadIdx.x < 11) w[threadIdx.x] = a.taps.w[threadIdx.x];
    const int c = blockIdx.z;
    const int tile_x0 = blockIdx.x * kBlock, tile_y0 = blockIdx.y * kBlock;
    const int tx = threadIdx.x % kBlock, ty = threadIdx.x / kBlock;
    const uint32_t px = tile_x0 + tx, py = tile_y0 + ty;
    const bool in = px < a.w && py < a.h;
    const size_t oidx = HWC4 ? ((size_t)py * a.w + px) * 4 + c : ((size_t)c * a.h + py) * a.w + px;
    if (c == 3) {  // alpha matching: |pred.a - gt.a|
        if (in) {
            float gc, ga;
            read_gt(a, 0, py, px, &gc, &ga);
            float v = fabsf(read_pred<HWC4>(a, 3, py, px) - ga);
            if (a.mask) v = v * ga;
            a.out[oidx] = v;
        }
        return;
    }
    if (a.ssim_w == 0.0f) {  // L1-only specialisation (lib.rs:232-276)
        if (in) {
            float ga;
            const float ge = gt_eff(a, c, py, px, &ga);
            float v = a.l1_w * fabsf(read_pred<HWC4>(a, c, py, px) - ge);
            if (a.mask) v = v * ga;
            a.out[oidx] = v;
        }
        return;
    }
    stage_tile<HWC4>(a, c, tile_x0, tile_y0, kShared, kHalo, s_x, s_y);
    __syncthreads();
    hblur_moments(s_x, s_y, kShared, kShared, kBlock, w, s_h);
    __syncthreads();
    float o[5];
    vblur5(s_h, kShared * kBlock, kBlock, ty + kHalo, tx, w, o);
    if (in) {
        const Ssim t = ssim_terms(o[0], o[1], o[2], o[3], o[4]);
        const int ci = (ty + kHalo) * kShared + tx + kHalo;
        const float l1 = fabsf(s_x[ci] - s_y[ci]);
        float v = a.l1_w * l1 + a.ssim_w * t.val;
        if (a.mask) {
            float gc, ga;
            read_gt(a, c, py, px, &gc, &ga);
            v = v * ga;
        }
        a.out[oidx] = v;
    }
}

// Shared buffers of the backward (and fused loss+backward), per channel:
//   s_x, s_y: staged pred / gt_eff planes, 36x36
//   s_h:      first horizontal blur, 5 planes of 36x26; later the second
//             horizontal blur, 3 planes of 26x16
//   s_p:      chain-weighted partials, 3 planes of 26x26
struct LossSmem {
    float x[kExtended * kExtended];
    float y[kExtended * kExtended];
    float h[5 * kExtended * kShared];
    float p[3 * kShared * kShared];
};

template <bool HWC4, bool FUSED>
__device__ __forceinline__ void loss_bwd_channel(const LossArgs& a, int c, int tile_x0, int tile_y0, const float* w,
                                                 LossSmem& S, float* s_val, float* grad_out, float* loss_out) {
    const int tx = threadIdx.x % kBlock, ty = threadIdx.x / kBlock;
    const uint32_t px = tile_x0 + tx, py = tile_y0 + ty;
    const bool in = px < a.w && py < a.h;
    stage_tile<HWC4>(a, c, tile_x0, tile_y0, kExtended, 2 * kHalo, S.x, S.y);
    __syncthreads();
    hblur_moments(S.x, S.y, kExtended, kExtended, kShared, w, S.h);
    __syncthreads();
    constexpr int kP = kShared * kShared;
    for (int tid = threadIdx.x; tid < kP; tid += blockDim.x) {
        const int pyl = tid / kShared, pxl = tid - pyl * kShared;
        float o[5];
        vblur5(S.h, kExtended * kShared, kShared, pyl + kHalo, pxl, w, o);
        const Ssim t = ssim_terms(o[0], o[1], o[2], o[3], o[4]);
        const int gy = tile_y0 + pyl - kHalo, gx = tile_x0 + pxl - kHalo;
        float chain = 0.0f;
        if (gy >= 0 && gx >= 0 && gy < (int)a.h && gx < (int)a.w) {
            chain = a.dl_dmap ? __ldg(a.dl_dmap + ((size_t)c * a.h + gy) * a.w + gx) : a.chain_const;
            if (a.mask) {
                float gc, ga;
                read_gt(a, c, gy, gx, &gc, &ga);
                chain = chain * ga;
            }
        }
        S.p[tid] = t.dmu1 * chain;
        S.p[kP + tid] = t.dsig1 * chain;
        S.p[2 * kP + tid] = t.dsig12 * chain;
        if (FUSED && pyl >= kHalo && pyl < kHalo + kBlock && pxl >= kHalo && pxl < kHalo + kBlock)
            s_val[(pyl - kHalo) * kBlock + (pxl - kHalo)] = t.val;
    }
    __syncthreads();
    // second horizontal blur: 26 rows x 16 columns x 3 planes
    constexpr int kQ = kShared * kBlock;
    for (int tid = threadIdx.x; tid < kQ; tid += blockDim.x) {
        const int ry = tid / kBlock, cx = tid - ry * kBlock;
        const int center = ry * kShared + cx + kHalo;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
        for (int d = 1; d < 6; ++d) {
            const float wd = w[5 - d];
            a0 += (S.p[center - d] + S.p[center + d]) * wd;
            a1 += (S.p[kP + center - d] + S.p[kP + center + d]) * wd;
            a2 += (S.p[2 * kP + center - d] + S.p[2 * kP + center + d]) * wd;
        }
        a0 += S.p[center] * w[5];
        a1 += S.p[kP + center] * w[5];
        a2 += S.p[2 * kP + center] * w[5];
        S.h[tid] = a0;
        S.h[kQ + tid] = a1;
        S.h[2 * kQ + tid] = a2;
    }
    __syncthreads();
    if (in) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
        const int ly = ty + kHalo;
#pragma unroll
        for (int d = 1; d < 6; ++d) {
            const float wd = w[5 - d];
            const int bt = (ly - d) * kBlock + tx, bb = (ly + d) * kBlock + tx;
            s0 += (S.h[bt] + S.h[bb]) * wd;
            s1 += (S.h[kQ + bt] + S.h[kQ + bb]) * wd;
            s2 += (S.h[2 * kQ + bt] + S.h[2 * kQ + bb]) * wd;
        }
        const int bc = ly * kBlock + tx;
        s0 += S.h[bc] * w[5];
        s1 += S.h[kQ + bc] * w[5];
        s2 += S.h[2 * kQ + bc] * w[5];
        const int ci = (ty + 2 * kHalo) * kExtended + tx + 2 * kHalo;
        const float p1 = S.x[ci];
        const float ge = S.y[ci];
        float gc_unused, ga = 1.0f;
        if (a.mask) read_gt(a, c, py, px, &gc_unused, &ga);
        const float sg = s0 + (2.0f * p1) * s1 + ge * s2;
        const float diff = p1 - ge;
        const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
        float chc = a.dl_dmap ? __ldg(a.dl_dmap + ((size_t)c * a.h + py) * a.w + px) : a.chain_const;
        if (a.mask) chc = chc * ga;
        *grad_out = a.ssim_w * sg + a.l1_w * sign * chc;
        if (FUSED) {
            float v = a.l1_w * fabsf(diff) + a.ssim_w * s_val[ty * kBlock + tx];
            if (a.mask) v = v * ga;
            *loss_out += v;
        }
    }
    __syncthreads();
}

template <bool HWC4>
__global__ void __launch_bounds__(256) loss_bwd_kernel(const __grid_constant__ LossArgs a) {
    __shared__ LossSmem S;
    __shared__ float w[11];
    if (threadIdx.x < 11) w[threadIdx.x] = a.taps.w[threadIdx.x];
    const int c = blockIdx.z;
    const int tile_x0 = blockIdx.x * kBlock, tile_y0 = blockIdx.y * kBlock;
    const int tx = threadIdx.x % kBlock, ty = threadIdx.x / kBlock;
    const uint32_t px = tile_x0 + tx, py = tile_y0 + ty;
    const bool in = px < a.w && py < a.h;
    const size_t idx = HWC4 ? ((size_t)py * a.w + px) * 4 + c : ((size_t)c * a.h + py) * a.w + px;
    if (c == 3 || a.ssim_w == 0.0f) {
        if (in) {
            float gc, ga;
            read_gt(a, c == 3 ? 0 : c, py, px, &gc, &ga);
            float ge = c == 3 ? ga : (a.composite ? gc + (1.0f - ga) * a.bg[c] : gc);
            const float diff = read_pred<HWC4>(a, c, py, px) - ge;
            const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            float ch = a.dl_dmap ? __ldg(a.dl_dmap + ((size_t)c * a.h + py) * a.w + px) : a.chain_const;
            if (a.mask) ch = ch * ga;
            a.out[idx] = (c == 3 ? 1.0f : a.l1_w) * sign * ch;
        }
        return;
    }
    __syncthreads();
    float g = 0.0f, unused = 0.0f;
    loss_bwd_channel<HWC4, false>(a, c, tile_x0, tile_y0, w, S, nullptr, &g, &unused);
    if (in) a.out[idx] = g;
}

// Training form: two launches over 32x32 output tiles, [H,W,4] in and out.
//
// loss_ssim_kernel stages a tile with a 5-pixel halo (42x42 samples, the three
// colour channels at once), blurs the five moments horizontally over the 42
// rows x 32 core columns and vertically over the 32x32 core, and writes for
// every image pixel the chain-weighted SSIM partials (d/d mu_x, d/d sigma_x^2,
// d/d sigma_xy, each times d loss / d map) with the loss summed per block.
// loss_grad_kernel (one channel per block) stages those partials over the same
// halo with 16-byte loads, blurs them horizontally then vertically, and forms
// each core pixel's gradient. Cutting at the partials leaves one halo per
// blur: each pass evaluates at most 1.31x its outputs, where one kernel doing
// all four passes needs 52x42 moment blurs and 42x42 SSIM values per 32x32
// tile. The partials (36 bytes per pixel) are written once and read back
// while still largely resident in L2.
//
// Quantities that are blurred alike travel in pairs through Blackwell's
// two-lane FP32 instructions (add / mul / fma .rn.f32x2, each lane rounded as
// the scalar instruction): the staged samples as (x, y), the moments as
// (mu_x, mu_y), (E[x^2], E[y^2]) and E[xy], the partials as
// (d/d mu_x, d/d sigma_x^2) and d/d sigma_xy. Blur passes run register sliding
// windows (a run of 8 outputs per thread horizontally, 4 vertically); planes
// have odd pitches, so lanes walking down a column (horizontal passes, one row
// per lane) or along a row (vertical passes) hit distinct banks. Tap and
// summation order per output are those of loss_bwd_channel: taps d = 1..5 as
// (left + right) * w[5-d], then the centre.
constexpr int kFT = 32;                        // output tile edge
constexpr int kFS = kFT + 2 * kHalo;           // 42: staged grid edge
constexpr int kFSP = kFS + 1;                  // 43: pitch of the staged planes
constexpr int kFHP = kFT + 1;                  // 33: pitch of the horizontal-blur planes
constexpr int kFThreads = 256;
constexpr int kRunH = 8;                       // outputs per thread, horizontal passes
constexpr int kRunV = 4;                       // outputs per thread, vertical passes
constexpr int kItemsH = kFS * (kFT / kRunH);   // 168 (row, run) items of a horizontal pass
static_assert(kFT * (kFT / kRunV) == kFThreads, "a vertical pass covers the tile once");
static_assert(kItemsH <= kFThreads, "a horizontal pass is one round");
constexpr int kFStage = kFS * kFSP;            // size of one staged plane
constexpr int kFH = kFS * kFHP;                // size of one horizontal-blur plane

// Two f32 lanes in one 64-bit register (low lane first).
typedef unsigned long long f2;
__device__ __forceinline__ f2 f2_pack(float lo, float hi) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float f2_lo(f2 v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo;
}
__device__ __forceinline__ float f2_hi(f2 v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return hi;
}
__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// Blur taps as lane pairs (w[k], w[k]).
struct Taps2 {
    f2 w[6];  // w[0..5] of the 11 symmetric taps
};
__device__ __forceinline__ Taps2 taps2(const LossTaps& t) {
    Taps2 r;
#pragma unroll
    for (int k = 0; k < 6; ++k) r.w[k] = f2_pack(t.w[k], t.w[k]);
    return r;
}

// Output j of the window v (centre v[j + 5]): (v[j+4] + v[j+6]) w4 first, then
// the taps d = 2..5, then the centre.
template <int N>
__device__ __forceinline__ void blur2(const f2* v, const Taps2& w, f2* out) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
        f2 acc = f2_mul(f2_add(v[j + 4], v[j + 6]), w.w[4]);
#pragma unroll
        for (int d = 2; d < 6; ++d) acc = f2_fma(f2_add(v[j + 5 - d], v[j + 5 + d]), w.w[5 - d], acc);
        out[j] = f2_fma(v[j + 5], w.w[5], acc);
    }
}
template <int N>
__device__ __forceinline__ void blur1(const float* v, const Taps2& w, float* out) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
        float acc = (v[j + 4] + v[j + 6]) * f2_lo(w.w[4]);
#pragma unroll
        for (int d = 2; d < 6; ++d) acc = __fmaf_rn(v[j + 5 - d] + v[j + 5 + d], f2_lo(w.w[5 - d]), acc);
        out[j] = __fmaf_rn(v[j + 5], f2_lo(w.w[5]), acc);
    }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float sum = 0.0f;
    if (threadIdx.x == 0)
        for (int k = 0; k < (int)(blockDim.x / 32); ++k) sum += red[k];
    return sum;
}

struct SsimSmem {
    f2 xy[3][kFStage];  // staged (prediction, effective ground truth) per channel, 42 x 42
    f2 m01[kFH];        // horizontal blur of one channel: (x, y)
    f2 m23[kFH];        //                                 (x^2, y^2)
    float m4[kFH];      //                                 x y
    float red[kFThreads / 32];
};

// Partial planes of channel c: (d/d mu_x, d/d sigma_x^2) pairs [H][pitch] at
// 3c planes, d/d sigma_xy [H][pitch] at 3c + 2 planes (plane = H * pitch floats).
__global__ void __launch_bounds__(kFThreads, 3)
    loss_ssim_kernel(const __grid_constant__ LossArgs a, float* __restrict__ planes, uint32_t pitch) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SsimSmem& S = *reinterpret_cast<SsimSmem*>(smem_raw);
    const Taps2 w = taps2(a.taps);
    const int x0 = blockIdx.x * kFT, y0 = blockIdx.y * kFT;
    // stage the 42x42 samples of all three channels (zero outside the image);
    // each thread issues all of its loads before its first store
    constexpr int kStageIters = (kFS * kFS + kFThreads - 1) / kFThreads;  // 7
    float4 pv[kStageIters];
    uint32_t gv[kStageIters];
#pragma unroll
    for (int i = 0; i < kStageIters; ++i) {
        const int t = threadIdx.x + i * kFThreads;
        const int ly = t / kFS, lx = t - ly * kFS;
        const int gy = y0 + ly - kHalo, gx = x0 + lx - kHalo;
        pv[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        gv[i] = 0u;
        if (t < kFS * kFS && gy >= 0 && gx >= 0 && gy < (int)a.h && gx < (int)a.w) {
            const size_t pid = (size_t)gy * a.w + gx;
            pv[i] = __ldg(reinterpret_cast<const float4*>(a.pred) + pid);
            gv[i] = __ldg(a.gt + pid);
        }
    }
#pragma unroll
    for (int i = 0; i < kStageIters; ++i) {
        const int t = threadIdx.x + i * kFThreads;
        if (t < kFS * kFS) {
            const int ly = t / kFS, lx = t - ly * kFS;
            const uint32_t v = gv[i];
            float g0 = (float)(v & 0xffu) * kInv255;
            float g1 = (float)((v >> 8u) & 0xffu) * kInv255;
            float g2 = (float)((v >> 16u) & 0xffu) * kInv255;
            if (a.composite) {
                // a zero sample outside the image stays zero
                const int gy = y0 + ly - kHalo, gx = x0 + lx - kHalo;
                const bool in = gy >= 0 && gx >= 0 && gy < (int)a.h && gx < (int)a.w;
                const float ta = in ? 1.0f - (float)(v >> 24u) * kInv255 : 0.0f;
                g0 = g0 + ta * a.bg[0];
                g1 = g1 + ta * a.bg[1];
                g2 = g2 + ta * a.bg[2];
            }
            const int o = ly * kFSP + lx;
            S.xy[0][o] = f2_pack(pv[i].x, g0);
            S.xy[1][o] = f2_pack(pv[i].y, g1);
            S.xy[2][o] = f2_pack(pv[i].z, g2);
        }
    }
    __syncthreads();
    // vertical-pass ownership: column col, rows r0 .. r0 + 3 of the tile
    const int col = threadIdx.x & (kFT - 1), r0 = (threadIdx.x / kFT) * kRunV;
    const size_t plane = (size_t)a.h * pitch;
    float loss = 0.0f;
    for (int c = 0; c < 3; ++c) {
        // horizontal moment blur: 42 rows x 32 columns, one row per lane
        if (threadIdx.x < kItemsH) {
            const int row = threadIdx.x % kFS, run = threadIdx.x / kFS;
            const f2* src = S.xy[c] + row * kFSP + run * kRunH;
            f2 v[kRunH + 10], o[kRunH];
#pragma unroll
            for (int k = 0; k < kRunH + 10; ++k) v[k] = src[k];
            const int hb = row * kFHP + run * kRunH;
            blur2<kRunH>(v, w, o);
#pragma unroll
            for (int j = 0; j < kRunH; ++j) S.m01[hb + j] = o[j];
            float t[kRunH + 10], ot[kRunH];
#pragma unroll
            for (int k = 0; k < kRunH + 10; ++k) t[k] = f2_lo(v[k]) * f2_hi(v[k]);
#pragma unroll
            for (int k = 0; k < kRunH + 10; ++k) v[k] = f2_mul(v[k], v[k]);
            blur2<kRunH>(v, w, o);
#pragma unroll
            for (int j = 0; j < kRunH; ++j) S.m23[hb + j] = o[j];
            blur1<kRunH>(t, w, ot);
#pragma unroll
            for (int j = 0; j < kRunH; ++j) S.m4[hb + j] = ot[j];
        }
        __syncthreads();
        // vertical blur + SSIM partials on the 32x32 core
        f2 mu[kRunV], sq[kRunV];
        float xy[kRunV];
        {
            f2 v[kRunV + 10];
#pragma unroll
            for (int t = 0; t < kRunV + 10; ++t) v[t] = S.m01[(r0 + t) * kFHP + col];
            blur2<kRunV>(v, w, mu);
#pragma unroll
            for (int t = 0; t < kRunV + 10; ++t) v[t] = S.m23[(r0 + t) * kFHP + col];
            blur2<kRunV>(v, w, sq);
            float u[kRunV + 10];
#pragma unroll
            for (int t = 0; t < kRunV + 10; ++t) u[t] = S.m4[(r0 + t) * kFHP + col];
            blur1<kRunV>(u, w, xy);
        }
#pragma unroll
        for (int j = 0; j < kRunV; ++j) {
            const uint32_t gx = x0 + col, gy = y0 + r0 + j;
            if (gx < a.w && gy < a.h) {
                const Ssim sm = ssim_terms(f2_lo(mu[j]), f2_lo(sq[j]), f2_hi(mu[j]), f2_hi(sq[j]), xy[j]);
                float chain = a.chain_const, ga = 1.0f;
                if (a.mask) {
                    ga = (float)(__ldg(a.gt + (size_t)gy * a.w + gx) >> 24u) * kInv255;
                    chain = chain * ga;
                }
                const size_t px = (size_t)gy * pitch + gx;
                reinterpret_cast<float2*>(planes + 3 * (size_t)c * plane)[px] =
                    make_float2(sm.dmu1 * chain, sm.dsig1 * chain);
                planes[(3 * (size_t)c + 2) * plane + px] = sm.dsig12 * chain;
                const f2 s = S.xy[c][(r0 + j + kHalo) * kFSP + col + kHalo];
                float v = a.l1_w * fabsf(f2_lo(s) - f2_hi(s)) + a.ssim_w * sm.val;
                if (a.mask) v = v * ga;
                loss += v;
            }
        }
        __syncthreads();  // the moment planes are rewritten by the next channel
    }
    const float sum = block_sum(loss, S.red);
    if (threadIdx.x == 0) a.block_loss[blockIdx.y * gridDim.x + blockIdx.x] = sum;
}

struct GradSmem {
    f2 p01[kFStage];   // staged (d/d mu_x, d/d sigma_x^2) partials, 42 x 42
    float p2[kFStage]; // staged d/d sigma_xy partials
    f2 q01[kFH];       // their horizontal blur, 42 x 32
    float q2[kFH];
};

// Grid (3, tiles x, tiles y): one colour channel per block, the three channel
// blocks of a tile adjacent in launch order (they read the same image and
// ground-truth lines); block c writes lane c of the [H,W,4] gradient (block 0
// also the zero alpha lane).
__global__ void __launch_bounds__(kFThreads, 5)
    loss_grad_kernel(const __grid_constant__ LossArgs a, const float* __restrict__ planes, uint32_t pitch) {
    __shared__ GradSmem S;
    const Taps2 w = taps2(a.taps);
    const int c = blockIdx.x;
    const int x0 = blockIdx.y * kFT, y0 = blockIdx.z * kFT;
    const int col = threadIdx.x & (kFT - 1), r0 = (threadIdx.x / kFT) * kRunV;
    const size_t plane = (size_t)a.h * pitch;
    const float* p01g = planes + 3 * (size_t)c * plane;
    const float* p2g = planes + (3 * (size_t)c + 2) * plane;
    // stage rows y0-5 .. y0+36 of both partial planes over the 48 columns
    // x0-8 .. x0+39 with 16-byte loads; staged column lx holds image column
    // x0 - 5 + lx, zero outside the image. The loads form 126 segments of 12:
    // segments 0-83 are the two halves of each row of pairs (two pixels per
    // load), 84-125 the rows of singles (four pixels per load); a round covers 21
    // segments, so rounds 0-3 read pairs and rounds 4-5 singles, uniformly per
    // warp. All loads of a thread are issued before its first store.
    constexpr int kQ4 = 12, kSegPerRound = kFThreads / kQ4;  // 21 (252 threads)
    constexpr int kPairSegs = 2 * kFS, kRounds = 3 * kFS / kSegPerRound;  // 84, 6
    static_assert(kPairSegs % kSegPerRound == 0 && 3 * kFS % kSegPerRound == 0, "uniform staging rounds");
    const int q4 = threadIdx.x % kQ4, sr = threadIdx.x / kQ4;
    const bool stager = sr < kSegPerRound;
    float4 v[kRounds];
#pragma unroll
    for (int i = 0; i < kRounds; ++i) {
        const int seg = sr + kSegPerRound * i;
        const bool pairs = i < kPairSegs / kSegPerRound;
        const int ly = pairs ? seg >> 1 : seg - kPairSegs;
        const int gx = pairs ? x0 - 8 + 24 * (seg & 1) + 2 * q4 : x0 - 8 + 4 * q4;
        const int gy = y0 + ly - kHalo;
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (stager && gy >= 0 && gy < (int)a.h && gx >= 0 && gx < (int)pitch)
            v[i] = pairs ? __ldg(reinterpret_cast<const float4*>(p01g + 2 * ((size_t)gy * pitch + gx)))
                         : __ldg(reinterpret_cast<const float4*>(p2g + (size_t)gy * pitch + gx));
    }
    if (stager) {
#pragma unroll
        for (int i = 0; i < kRounds; ++i) {
            const int seg = sr + kSegPerRound * i;
            if (i < kPairSegs / kSegPerRound) {
                const int ly = seg >> 1, lx = 24 * (seg & 1) + 2 * q4 - 3;
                const int gx = x0 - 5 + lx;
                f2* dst = S.p01 + ly * kFSP;
                if (lx >= 0 && lx < kFS) dst[lx] = gx < (int)a.w ? f2_pack(v[i].x, v[i].y) : 0ull;
                if (lx + 1 >= 0 && lx + 1 < kFS) dst[lx + 1] = gx + 1 < (int)a.w ? f2_pack(v[i].z, v[i].w) : 0ull;
            } else {
                const int ly = seg - kPairSegs, lx = 4 * q4 - 3;
                const int gx = x0 - 5 + lx;
                const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
                float* dst = S.p2 + ly * kFSP;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (lx + u >= 0 && lx + u < kFS) dst[lx + u] = gx + u < (int)a.w ? e[u] : 0.0f;
            }
        }
    }
    __syncthreads();
    // horizontal blur of the partials: 42 rows x 32 columns, one row per lane
    if (threadIdx.x < kItemsH) {
        const int row = threadIdx.x % kFS, run = threadIdx.x / kFS;
        const int sb = row * kFSP + run * kRunH, hb = row * kFHP + run * kRunH;
        f2 t2[kRunH + 10], o2[kRunH];
#pragma unroll
        for (int u = 0; u < kRunH + 10; ++u) t2[u] = S.p01[sb + u];
        blur2<kRunH>(t2, w, o2);
#pragma unroll
        for (int j = 0; j < kRunH; ++j) S.q01[hb + j] = o2[j];
        float t1[kRunH + 10], o1[kRunH];
#pragma unroll
        for (int u = 0; u < kRunH + 10; ++u) t1[u] = S.p2[sb + u];
        blur1<kRunH>(t1, w, o1);
#pragma unroll
        for (int j = 0; j < kRunH; ++j) S.q2[hb + j] = o1[j];
    }
    __syncthreads();
    // vertical blur -> gradient of this thread's four pixels (their prediction
    // and ground truth are loaded first, so that the loads overlap the blur)
    float p_px[kRunV];
    uint32_t gt_px[kRunV];
#pragma unroll
    for (int j = 0; j < kRunV; ++j) {
        const uint32_t gx = x0 + col, gy = y0 + r0 + j;
        const bool in = gx < a.w && gy < a.h;
        p_px[j] = in ? read_pred<true>(a, c, gy, gx) : 0.0f;
        gt_px[j] = in ? __ldg(a.gt + (size_t)gy * a.w + gx) : 0u;
    }
    f2 s01[kRunV];
    float s2[kRunV];
    {
        f2 t2[kRunV + 10];
#pragma unroll
        for (int u = 0; u < kRunV + 10; ++u) t2[u] = S.q01[(r0 + u) * kFHP + col];
        blur2<kRunV>(t2, w, s01);
        float t1[kRunV + 10];
#pragma unroll
        for (int u = 0; u < kRunV + 10; ++u) t1[u] = S.q2[(r0 + u) * kFHP + col];
        blur1<kRunV>(t1, w, s2);
    }
#pragma unroll
    for (int j = 0; j < kRunV; ++j) {
        const uint32_t gx = x0 + col, gy = y0 + r0 + j;
        if (gx < a.w && gy < a.h) {
            const float p1 = p_px[j];
            const float ga = (float)(gt_px[j] >> 24u) * kInv255;
            float ge = (float)((gt_px[j] >> (8u * c)) & 0xffu) * kInv255;
            if (a.composite) ge = ge + (1.0f - ga) * a.bg[c];
            const float sg = f2_lo(s01[j]) + (2.0f * p1) * f2_hi(s01[j]) + ge * s2[j];
            const float diff = p1 - ge;
            const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            float chc = a.chain_const;
            if (a.mask) chc = chc * ga;
            float* dst = a.out + ((size_t)gy * a.w + gx) * 4;
            dst[c] = a.ssim_w * sg + a.l1_w * sign * chc;
            if (c == 0) dst[3] = 0.0f;
        }
    }
}

// L1-only training form (ssim weight 0): one thread per pixel, all channels.
constexpr int kL1Threads = 256;
__global__ void __launch_bounds__(kL1Threads) loss_l1_fused_kernel(const __grid_constant__ LossArgs a) {
    __shared__ float red[kL1Threads / 32];
    const size_t pid = (size_t)blockIdx.x * kL1Threads + threadIdx.x;
    float loss = 0.0f;
    if (pid < (size_t)a.w * a.h) {
        const uint32_t py = (uint32_t)(pid / a.w), px = (uint32_t)(pid - (size_t)py * a.w);
        float g[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float ga;
            const float ge = gt_eff(a, c, py, px, &ga);
            const float diff = read_pred<true>(a, c, py, px) - ge;
            const float sign = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            float ch = a.chain_const;
            float v = a.l1_w * fabsf(diff);
            if (a.mask) {
                ch = ch * ga;
                v = v * ga;
            }
            g[c] = a.l1_w * sign * ch;
            loss += v;
        }
        reinterpret_cast<float4*>(a.out)[pid] = make_float4(g[0], g[1], g[2], 0.0f);
    }
    const float sum = block_sum(loss, red);
    if (threadIdx.x == 0) a.block_loss[blockIdx.x] = sum;
}

__global__ void __launch_bounds__(1024) loss_mean_kernel(const float* partials, uint32_t count, double inv_n, float* out) {
    __shared__ double s[32];
    double acc = 0.0;
    for (uint32_t i = threadIdx.x; i < count; i += blockDim.x) acc += (double)partials[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < (int)(blockDim.x / 32); ++k) t += s[k];
        *out = (float)(t * inv_n);
    }
}

LossTaps make_taps() {
    // 11 taps at sigma 1.5 normalised to 1, computed in float as the reference
    // does when it builds the kernel (lib.rs:87-100).
    LossTaps t;
    float sum = 0.0f;
    const float s = 1.5f;
    for (int i = 0; i < 11; ++i) {
        const float x = (float)i - 5.0f;
        t.w[i] = std::exp(-x * x / (2.0f * s * s));
        sum += t.w[i];
    }
    for (int i = 0; i < 11; ++i) t.w[i] /= sum;
    return t;
}

LossArgs make_args(const bsx_loss_cfg* cfg, const float* pred, const uint32_t* gt, uint32_t w, uint32_t h) {
    LossArgs a;
    a.pred = pred;
    a.gt = gt;
    a.dl_dmap = nullptr;
    a.chain_const = 0.0f;
    a.out = nullptr;
    a.block_loss = nullptr;
    a.w = w;
    a.h = h;
    a.l1_w = cfg->l1_weight;
    a.ssim_w = cfg->ssim_weight;
    a.composite = cfg->composite_bg;
    a.mask = cfg->mask;
    a.bg[0] = cfg->bg[0];
    a.bg[1] = cfg->bg[1];
    a.bg[2] = cfg->bg[2];
    a.taps = make_taps();
    return a;
}

}  // namespace

}  // namespace bsx

using namespace bsx;

extern "C" {

bsx_status bsx_loss_fwd(bsx_ctx* ctx, const float* d_pred, const uint32_t* d_gt, uint32_t w, uint32_t h,
                        uint32_t channels, const bsx_loss_cfg* cfg, float* d_map) {
    if (!ctx || !d_pred || !d_gt || !cfg || !d_map || w == 0 || h == 0) return BSX_ERR_INVALID_ARG;
    if (channels != 3 && channels != 4) return fail(ctx, BSX_ERR_SHAPE, "loss expects 3 or 4 channels");
    cudaSetDevice(ctx->device);
    LossArgs a = make_args(cfg, d_pred, d_gt, w, h);
    a.out = d_map;
    dim3 grid((w + kBlock - 1) / kBlock, (h + kBlock - 1) / kBlock, channels);
    prof_begin(ctx);
    loss_fwd_kernel<false><<<grid, 256, 0, ctx->stream>>>(a);
    return post_launch(ctx, "loss_fwd_kernel");
}

bsx_status bsx_loss_bwd(bsx_ctx* ctx, const float* d_pred, const uint32_t* d_gt, uint32_t w, uint32_t h,
                        uint32_t channels, const bsx_loss_cfg* cfg, const float* d_dl_dmap, float* d_dl_dpred) {
    if (!ctx || !d_pred || !d_gt || !cfg || !d_dl_dmap || !d_dl_dpred || w == 0 || h == 0) return BSX_ERR_INVALID_ARG;
    if (channels != 3 && channels != 4) return fail(ctx, BSX_ERR_SHAPE, "loss expects 3 or 4 channels");
    cudaSetDevice(ctx->device);
    LossArgs a = make_args(cfg, d_pred, d_gt, w, h);
    a.dl_dmap = d_dl_dmap;
    a.out = d_dl_dpred;
    dim3 grid((w + kBlock - 1) / kBlock, (h + kBlock - 1) / kBlock, channels);
    prof_begin(ctx);
    loss_bwd_kernel<false><<<grid, 256, 0, ctx->stream>>>(a);
    return post_launch(ctx, "loss_bwd_kernel");
}

bsx_status bsx_loss_fused(bsx_ctx* ctx, const float* d_image, const uint32_t* d_gt, uint32_t w, uint32_t h,
                          const bsx_loss_cfg* cfg, float* d_loss_mean, float* d_v_output) {
    if (!ctx || !d_image || !d_gt || !cfg || !d_loss_mean || !d_v_output || w == 0 || h == 0) return BSX_ERR_INVALID_ARG;
    if (((uintptr_t)d_image | (uintptr_t)d_v_output) % 16) return fail(ctx, BSX_ERR_INVALID_ARG, "[H,W,4] buffers must be 16-byte aligned");
    cudaSetDevice(ctx->device);
    LossArgs a = make_args(cfg, d_image, d_gt, w, h);
    const double n = 3.0 * (double)w * (double)h;
    a.chain_const = (float)(1.0 / n);
    a.out = d_v_output;
    const bool ssim = cfg->ssim_weight != 0.0f;
    const dim3 grid = ssim ? dim3((w + kFT - 1) / kFT, (h + kFT - 1) / kFT, 1)
                           : dim3((uint32_t)(((size_t)w * h + kL1Threads - 1) / kL1Threads), 1, 1);
    const uint32_t blocks = grid.x * grid.y;
    bsx_status s = ensure(ctx, ctx->loss_partials, (size_t)blocks * 4);
    if (s != BSX_OK) return s;
    a.block_loss = ctx->loss_partials.as<float>();
    if (ssim) {
        const uint32_t pitch = (w + 3u) & ~3u;
        s = ensure(ctx, ctx->loss_planes, 9 * (size_t)h * pitch * 4);
        if (s != BSX_OK) return s;
        constexpr size_t kSsimSmem = sizeof(SsimSmem);
        static_assert(kSsimSmem <= 227 * 1024, "SSIM pass shared memory");
        s = check_cuda(ctx, cudaFuncSetAttribute(loss_ssim_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kSsimSmem),
                       "cudaFuncSetAttribute (SSIM pass)");
        if (s != BSX_OK) return s;
        float* planes = ctx->loss_planes.as<float>();
        prof_begin(ctx);
        loss_ssim_kernel<<<grid, kFThreads, kSsimSmem, ctx->stream>>>(a, planes, pitch);
        if ((s = post_launch(ctx, "loss_ssim_kernel")) != BSX_OK) return s;
        prof_begin(ctx);
        loss_grad_kernel<<<dim3(3, grid.x, grid.y), kFThreads, 0, ctx->stream>>>(a, planes, pitch);
        if ((s = post_launch(ctx, "loss_grad_kernel")) != BSX_OK) return s;
    } else {
        prof_begin(ctx);
        loss_l1_fused_kernel<<<grid, kL1Threads, 0, ctx->stream>>>(a);
        if ((s = post_launch(ctx, "loss_l1_fused_kernel")) != BSX_OK) return s;
    }
    prof_begin(ctx);
    loss_mean_kernel<<<1, 1024, 0, ctx->stream>>>(a.block_loss, blocks, 1.0 / n, d_loss_mean);
    return post_launch(ctx, "loss_mean_kernel");
}

}  // extern "C"
