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
// The training form (loss_fused_kernel) reads the rasterizer's [H,W,4] image
// directly, loops over the three colour channels inside one block, uses the
// constant chain 1/(3HW) of a mean reduction, writes the gradient straight
// into the [H,W,4] v_output layout the raster backward consumes (alpha lane
// 0), and emits per-block loss sums that a second tiny kernel reduces in a
// fixed order. This removes the reference's permute/contiguous copies, the
// separate mean kernel and the zero-fill of the gradient image.
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
    Ssim r;
    r.val = bsx_clamp((ct * dt) / (a * b), -1.0f, 1.0f);
    const float inv_ab = 1.0f / (a * b);
    const float cd = ct * dt * inv_ab;
    const bool clamped = cd < -1.0f || cd > 1.0f;
    r.dmu1 = clamped ? 0.0f : 2.0f * mu2 * inv_ab * (dt - ct) - 2.0f * mu1 * cd * (1.0f / a - 1.0f / b);
    r.dsig1 = clamped ? 0.0f : -cd / b;
    r.dsig12 = clamped ? 0.0f : 2.0f * ct * inv_ab;
    return r;
}

// Stage (pred, gt_eff) of an (ext x ext) region starting `halo` pixels before
// the tile into s[ext*ext*2]; out-of-image samples are zero.
template <bool HWC4>
__device__ __forceinline__ void stage_tile(const LossArgs& a, int c, int tile_x0, int tile_y0, int ext, int halo,
                                           float* s) {
    for (int tid = threadIdx.x; tid < ext * ext; tid += blockDim.x) {
        const int ly = tid / ext, lx = tid % ext;
        const int gy = tile_y0 + ly - halo, gx = tile_x0 + lx - halo;
        float pv = 0.0f, ge = 0.0f;
        if (gy >= 0 && gx >= 0 && gy < (int)a.h && gx < (int)a.w) {
            pv = read_pred<HWC4>(a, c, gy, gx);
            float ga;
            ge = gt_eff(a, c, gy, gx, &ga);
        }
        s[tid * 2] = pv;
        s[tid * 2 + 1] = ge;
    }
}

// Horizontal moment blur: rows [0,rows) of the staged region, output columns
// [0,cols) centred at staged column col + 5.
__device__ __forceinline__ void hblur_moments(const float* s, int ext, int rows, int cols, const float* w, float* o) {
    for (int tid = threadIdx.x; tid < rows * cols; tid += blockDim.x) {
        const int ry = tid / cols, cx = tid % cols;
        const int center = cx + kHalo;
        float sx = 0.f, sx2 = 0.f, sy = 0.f, sy2 = 0.f, sxy = 0.f;
#pragma unroll
        for (int d = 1; d < 6; ++d) {
            const float wd = w[5 - d];
            const int il = (ry * ext + center - d) * 2, ir = (ry * ext + center + d) * 2;
            const float xl = s[il], yl = s[il + 1], xr = s[ir], yr = s[ir + 1];
            sx += (xl + xr) * wd;
            sx2 += (xl * xl + xr * xr) * wd;
            sy += (yl + yr) * wd;
            sy2 += (yl * yl + yr * yr) * wd;
            sxy += (xl * yl + xr * yr) * wd;
        }
        const int ic = (ry * ext + center) * 2;
        const float xc = s[ic], yc = s[ic + 1], wc = w[5];
        sx += xc * wc;
        sx2 += xc * xc * wc;
        sy += yc * wc;
        sy2 += yc * yc * wc;
        sxy += xc * yc * wc;
        float* dst = o + (ry * cols + cx) * 5;
        dst[0] = sx;
        dst[1] = sx2;
        dst[2] = sy;
        dst[3] = sy2;
        dst[4] = sxy;
    }
}

__device__ __forceinline__ void vblur5(const float* hb, int cols, int center_row, int col, const float* w, float o[5]) {
#pragma unroll
    for (int k = 0; k < 5; ++k) o[k] = 0.0f;
#pragma unroll
    for (int d = 1; d < 6; ++d) {
        const float wd = w[5 - d];
        const float* t = hb + ((center_row - d) * cols + col) * 5;
        const float* b = hb + ((center_row + d) * cols + col) * 5;
#pragma unroll
        for (int k = 0; k < 5; ++k) o[k] += (t[k] + b[k]) * wd;
    }
    const float* cc = hb + (center_row * cols + col) * 5;
#pragma unroll
    for (int k = 0; k < 5; ++k) o[k] += cc[k] * w[5];
}

// Forward loss map, reference layout [C,H,W]; grid (tx, ty, C).
template <bool HWC4>
__global__ void __launch_bounds__(256) loss_fwd_kernel(const LossArgs a) {
    __shared__ float s_tile[kShared * kShared * 2];
    __shared__ float s_h[kShared * kBlock * 5];
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
    stage_tile<HWC4>(a, c, tile_x0, tile_y0, kShared, kHalo, s_tile);
    __syncthreads();
    hblur_moments(s_tile, kShared, kShared, kBlock, w, s_h);
    __syncthreads();
    float o[5];
    vblur5(s_h, kBlock, ty + kHalo, tx, w, o);
    if (in) {
        const Ssim t = ssim_terms(o[0], o[1], o[2], o[3], o[4]);
        const int ci = ((ty + kHalo) * kShared + tx + kHalo) * 2;
        const float l1 = fabsf(s_tile[ci] - s_tile[ci + 1]);
        float v = a.l1_w * l1 + a.ssim_w * t.val;
        if (a.mask) {
            float gc, ga;
            read_gt(a, c, py, px, &gc, &ga);
            v = v * ga;
        }
        a.out[oidx] = v;
    }
}

// Backward (and fused loss+backward). Shared layout per channel:
//   s_a: staged (pred, gt_eff), 36x36x2
//   s_b: first horizontal blur 36x26x5, later second horizontal blur 26x16x3
//   s_p: chain-weighted partials 26x26x3
template <bool HWC4, bool FUSED>
__device__ __forceinline__ void loss_bwd_channel(const LossArgs& a, int c, int tile_x0, int tile_y0, const float* w,
                                                 float* s_a, float* s_b, float* s_p, float* s_val, float* grad_out,
                                                 float* loss_out) {
    const int tx = threadIdx.x % kBlock, ty = threadIdx.x / kBlock;
    const uint32_t px = tile_x0 + tx, py = tile_y0 + ty;
    const bool in = px < a.w && py < a.h;
    stage_tile<HWC4>(a, c, tile_x0, tile_y0, kExtended, 2 * kHalo, s_a);
    __syncthreads();
    hblur_moments(s_a, kExtended, kExtended, kShared, w, s_b);
    __syncthreads();
    for (int tid = threadIdx.x; tid < kShared * kShared; tid += blockDim.x) {
        const int pyl = tid / kShared, pxl = tid % kShared;
        float o[5];
        vblur5(s_b, kShared, pyl + kHalo, pxl, w, o);
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
        s_p[tid * 3] = t.dmu1 * chain;
        s_p[tid * 3 + 1] = t.dsig1 * chain;
        s_p[tid * 3 + 2] = t.dsig12 * chain;
        if (FUSED && pyl >= kHalo && pyl < kHalo + kBlock && pxl >= kHalo && pxl < kHalo + kBlock)
            s_val[(pyl - kHalo) * kBlock + (pxl - kHalo)] = t.val;
    }
    __syncthreads();
    // second horizontal blur: 26 rows x 16 columns x 3
    for (int tid = threadIdx.x; tid < kShared * kBlock; tid += blockDim.x) {
        const int ry = tid / kBlock, cx = tid % kBlock;
        const int center = cx + kHalo;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
        for (int d = 1; d < 6; ++d) {
            const float wd = w[5 - d];
            const int il = (ry * kShared + center - d) * 3, ir = (ry * kShared + center + d) * 3;
            a0 += (s_p[il] + s_p[ir]) * wd;
            a1 += (s_p[il + 1] + s_p[ir + 1]) * wd;
            a2 += (s_p[il + 2] + s_p[ir + 2]) * wd;
        }
        const int ic = (ry * kShared + center) * 3;
        a0 += s_p[ic] * w[5];
        a1 += s_p[ic + 1] * w[5];
        a2 += s_p[ic + 2] * w[5];
        s_b[tid * 3] = a0;
        s_b[tid * 3 + 1] = a1;
        s_b[tid * 3 + 2] = a2;
    }
    __syncthreads();
    if (in) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
        const int ly = ty + kHalo;
#pragma unroll
        for (int d = 1; d < 6; ++d) {
            const float wd = w[5 - d];
            const int bt = ((ly - d) * kBlock + tx) * 3, bb = ((ly + d) * kBlock + tx) * 3;
            s0 += (s_b[bt] + s_b[bb]) * wd;
            s1 += (s_b[bt + 1] + s_b[bb + 1]) * wd;
            s2 += (s_b[bt + 2] + s_b[bb + 2]) * wd;
        }
        const int bc = (ly * kBlock + tx) * 3;
        s0 += s_b[bc] * w[5];
        s1 += s_b[bc + 1] * w[5];
        s2 += s_b[bc + 2] * w[5];
        const float p1 = read_pred<HWC4>(a, c, py, px);
        float ga;
        const float ge = gt_eff(a, c, py, px, &ga);
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
__global__ void __launch_bounds__(256) loss_bwd_kernel(const LossArgs a) {
    __shared__ float s_a[kExtended * kExtended * 2];
    __shared__ float s_b[kExtended * kShared * 5];
    __shared__ float s_p[kShared * kShared * 3];
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
    loss_bwd_channel<HWC4, false>(a, c, tile_x0, tile_y0, w, s_a, s_b, s_p, nullptr, &g, &unused);
    if (in) a.out[idx] = g;
}

// Training form: three colour channels per block, [H,W,4] in and out.
__global__ void __launch_bounds__(256) loss_fused_kernel(const LossArgs a) {
    __shared__ float s_a[kExtended * kExtended * 2];
    __shared__ float s_b[kExtended * kShared * 5];
    __shared__ float s_p[kShared * kShared * 3];
    __shared__ float s_val[kBlock * kBlock];
    __shared__ float w[11];
    __shared__ float s_red[8];
    if (threadIdx.x < 11) w[threadIdx.x] = a.taps.w[threadIdx.x];
    __syncthreads();
    const int tile_x0 = blockIdx.x * kBlock, tile_y0 = blockIdx.y * kBlock;
    const int tx = threadIdx.x % kBlock, ty = threadIdx.x / kBlock;
    const uint32_t px = tile_x0 + tx, py = tile_y0 + ty;
    float g[3] = {0.f, 0.f, 0.f};
    float loss = 0.0f;
    if (a.ssim_w == 0.0f) {
        if (px < a.w && py < a.h) {
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
        }
    } else {
        for (int c = 0; c < 3; ++c)
            loss_bwd_channel<true, true>(a, c, tile_x0, tile_y0, w, s_a, s_b, s_p, s_val, &g[c], &loss);
    }
    if (px < a.w && py < a.h)
        reinterpret_cast<float4*>(a.out)[(size_t)py * a.w + px] = make_float4(g[0], g[1], g[2], 0.0f);
    // block loss sum (fixed order)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = loss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int k = 0; k < 8; ++k) s += s_red[k];
        a.block_loss[blockIdx.y * gridDim.x + blockIdx.x] = s;
    }
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
    dim3 grid((w + kBlock - 1) / kBlock, (h + kBlock - 1) / kBlock, 1);
    const uint32_t blocks = grid.x * grid.y;
    bsx_status s = ensure(ctx, ctx->loss_partials, (size_t)blocks * 4);
    if (s != BSX_OK) return s;
    LossArgs a = make_args(cfg, d_image, d_gt, w, h);
    const double n = 3.0 * (double)w * (double)h;
    a.chain_const = (float)(1.0 / n);
    a.out = d_v_output;
    a.block_loss = ctx->loss_partials.as<float>();
    prof_begin(ctx);
    loss_fused_kernel<<<grid, 256, 0, ctx->stream>>>(a);
    s = post_launch(ctx, "loss_fused_kernel");
    if (s != BSX_OK) return s;
    prof_begin(ctx);
    loss_mean_kernel<<<1, 1024, 0, ctx->stream>>>(a.block_loss, blocks, 1.0 / n, d_loss_mean);
    return post_launch(ctx, "loss_mean_kernel");
}

}  // extern "C"
