/*
 * bsx_fmath.h - deterministic float32 elementary functions shared by the
 * sm_100a kernels and host code.
 *
 * Why this exists: the splat pipeline takes discrete decisions from float
 * predicates (cull on opacity, intersection counts from ln(255*opacity),
 * the alpha >= 1/255 cutoff, the T <= 1e-4 early-out). To make those
 * decisions identical on the GPU and on a CPU restatement, every
 * transcendental on the path is evaluated with the SAME sequence of IEEE
 * operations on both sides: + - * / sqrt (correctly rounded by IEEE 754 on
 * both processors), explicit fused multiply-add (also correctly rounded on
 * both), and integer bit manipulation.
 *
 * The reference evaluates exp/ln with its shading language's builtins,
 * whose accuracy its own tests bound only by tolerance; the functions here
 * take that role.
 *
 * Methods (published, restated here; coefficients derived from the math):
 *  - exp: Cody & Waite argument reduction x = k*ln2 + r with ln2 split into
 *    a 15-bit head (exact products for |k| <= 255) and a tail, followed by
 *    the degree-7 Taylor polynomial of e^r on |r| <= ln2/2 (truncation error
 *    r^8/8! < 5.3e-9 relative), then exact scaling by 2^k. The rasterizers'
 *    exp (bsx_expf_raster) trades a little accuracy for fewer operations on
 *    its bounded domain.
 *  - ln: x = m * 2^e with m in [sqrt(1/2), sqrt(2)), s = (m-1)/(m+1),
 *    ln(m) = 2*atanh(s) = 2s(1 + s^2/3 + s^4/5 + ... + s^10/11)
 *    (|s| <= 0.1716, truncation < 2e-10 relative), plus e*ln2.
 * Accuracy against the C library is checked by the CPU test-suite.
 *
 * Compile the including translation units without floating-point
 * contraction (nvcc -fmad=false, gcc -ffp-contract=off) so that expressions
 * are evaluated exactly as written.
 */
#ifndef BSX_FMATH_H
#define BSX_FMATH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define BSX_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#include <string.h>
#define BSX_HD static inline
#endif

BSX_HD float bsx_bits_to_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
#endif
}

BSX_HD uint32_t bsx_f32_to_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    return u;
#endif
}

/* Correctly rounded a*b+c on both processors. */
BSX_HD float bsx_fma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return fmaf(a, b, c);
#endif
}

/* Round to nearest integer, ties to even (IEEE default mode on both). */
BSX_HD float bsx_rint(float x) {
#if defined(__CUDA_ARCH__)
    return rintf(x);
#else
    return nearbyintf(x);
#endif
}

/* IEEE minNum/maxNum: a NaN operand yields the other operand. */
BSX_HD float bsx_min(float a, float b) { return fminf(a, b); }
BSX_HD float bsx_max(float a, float b) { return fmaxf(a, b); }
BSX_HD float bsx_clamp(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

/* 2^k as a float for k in [-126, 127]. */
BSX_HD float bsx_pow2i(int k) { return bsx_bits_to_f32((uint32_t)(k + 127) << 23); }

/* Bit-level finiteness test (exponent field not all ones). */
BSX_HD int bsx_is_finite(float x) { return ((bsx_f32_to_bits(x) >> 23) & 0xFFu) != 0xFFu; }

/* exp(x) in float32. NaN propagates; overflow gives +inf; deep underflow 0. */
BSX_HD float bsx_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return bsx_bits_to_f32(0x7f800000u);
    if (x < -103.97209167480469f) return 0.0f;
    const float kLog2e = 1.4426950216293335f;
    const float kLn2Hi = 0.693145751953125f;    /* 0x3f317200 */
    const float kLn2Lo = 1.428606765330187e-06f; /* 0x35bfbe8e */
    float k = bsx_rint(x * kLog2e);
    float r = bsx_fma(-k, kLn2Hi, x);
    r = bsx_fma(-k, kLn2Lo, r);
    float p = 0.00019841270113829523f;       /* 1/7! */
    p = bsx_fma(p, r, 0.0013888889225199819f); /* 1/6! */
    p = bsx_fma(p, r, 0.008333333767950535f);  /* 1/5! */
    p = bsx_fma(p, r, 0.0416666679084301f);    /* 1/4! */
    p = bsx_fma(p, r, 0.1666666716337204f);    /* 1/3! */
    p = bsx_fma(p, r, 0.5f);
    p = bsx_fma(p, r, 1.0f);
    p = bsx_fma(p, r, 1.0f);
    int ki = (int)k;
    if (ki >= -126 && ki <= 127) return p * bsx_pow2i(ki);
    if (ki > 127) return (p * bsx_pow2i(127)) * 2.0f;
    return (p * bsx_pow2i(ki + 64)) * 5.421010862427522e-20f; /* 2^-64 */
}

/* exp(x) for the rasterizers' Gaussian falloff, x in [-87, 0] (there e^x is
 * a normal float; the rasterizers only evaluate x >= -(ln(255) + 1)):
 *  - k = rint(x*log2e) by the round-to-integer constant 1.5*2^23 added in the
 *    same fused multiply-add, then r = x - k*ln2 with one float ln2 (for
 *    |k| <= 24, i.e. x >= -16, the reduction error is below 0.4 ulp);
 *  - e^r on |r| <= ln2/2 by a degree-6 polynomial whose coefficients come
 *    from a Remez exchange for relative error, rounded to float (minimax
 *    error 1.9e-9 before rounding);
 *  - p*2^k by adding k to p's exponent field: the low bits of
 *    x*log2e + 1.5*2^23 hold k in two's complement, and the constant's own
 *    mantissa bits vanish when shifted left by 23; the result is normal on
 *    the domain, so the integer add equals the exact product.
 * Error against the exact exponential: at most 1.4 ulp on [-16, 0] (every
 * float checked; 99% of them below 0.5 ulp), at most 4.5 ulp on [-87, -16].
 * The CPU test-suite checks a sweep of the domain against the C library. */
BSX_HD float bsx_expf_raster(float x) {
    const float kLog2e = 1.4426950216293335f;
    const float kLn2 = 0.693147182464599609375f;
    const float kRound = 12582912.0f; /* 1.5 * 2^23 */
    const float tk = bsx_fma(x, kLog2e, kRound);
    const float k = tk - kRound;
    const float r = bsx_fma(-k, kLn2, x);
    float p = 0.0013836835278198123f;
    p = bsx_fma(p, r, 0.008374824188649654f);
    p = bsx_fma(p, r, 0.04166822507977486f);
    p = bsx_fma(p, r, 0.16666419804096222f);
    p = bsx_fma(p, r, 0.49999991059303284f);
    p = bsx_fma(p, r, 1.0f);
    p = bsx_fma(p, r, 1.0f);
    return bsx_bits_to_f32(bsx_f32_to_bits(p) + (bsx_f32_to_bits(tk) << 23));
}

/* The rasterizers' sigma = 0.5 (c00 dx^2 + c11 dy^2) + c01 dx dy
 * (brush-cube/src/lib.rs:634-638) as one fixed sequence of roundings, shared
 * by the forward and backward kernels and their CPU restatement:
 *   hxx = 0.5 ((c00 dx) dx),  sigma = fma(c01 dx, dy, fma((0.5 c11) dy, dy, hxx)).
 * Halving is exact, so this is the expression with fused products; hxx and
 * c01 dx depend only on the column and are shared by pixels that have it. */
BSX_HD float bsx_sigma_hxx(float c00, float dx) { return 0.5f * ((c00 * dx) * dx); }
BSX_HD float bsx_sigma_row(float hxx, float xy, float hc11, float dy) {
    return bsx_fma(xy, dy, bsx_fma(hc11 * dy, dy, hxx));
}
BSX_HD float bsx_raster_sigma(float c00, float c01, float c11, float dx, float dy) {
    return bsx_sigma_row(bsx_sigma_hxx(c00, dx), c01 * dx, 0.5f * c11, dy);
}

/* Natural logarithm in float32. */
BSX_HD float bsx_logf(float x) {
    if (x != x) return x;
    if (x < 0.0f) return bsx_bits_to_f32(0x7fc00000u);
    if (x == 0.0f) return bsx_bits_to_f32(0xff800000u);
    uint32_t b = bsx_f32_to_bits(x);
    if (b >= 0x7f800000u) return x; /* +inf */
    int e = 0;
    if (b < 0x00800000u) { /* subnormal: scale into the normal range */
        x = x * 8388608.0f;  /* 2^23, exact */
        b = bsx_f32_to_bits(x);
        e = -23;
    }
    e += (int)(b >> 23) - 127;
    float m = bsx_bits_to_f32((b & 0x007fffffu) | 0x3f800000u);
    if (m > 1.4142135381698608f) {
        m = m * 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    float s2 = s * s;
    float q = 0.09090909361839294f;             /* 1/11 */
    q = bsx_fma(q, s2, 0.1111111119389534f);    /* 1/9 */
    q = bsx_fma(q, s2, 0.1428571492433548f);    /* 1/7 */
    q = bsx_fma(q, s2, 0.20000000298023224f);   /* 1/5 */
    q = bsx_fma(q, s2, 0.3333333432674408f);    /* 1/3 */
    float t = s + s;
    float lnm = bsx_fma(t * s2, q, t);
    float ef = (float)e;
    return bsx_fma(ef, 0.693145751953125f, bsx_fma(ef, 1.428606765330187e-06f, lnm));
}

/* atan(t) for t in [0, 1]. Above tan(pi/12) the argument is reduced by the
 * addition formula atan(t) = pi/6 + atan((t - c) / (1 + t c)), c = 1/sqrt(3),
 * which leaves |t'| <= tan(pi/12) = 0.268; then the Maclaurin series
 * t - t^3/3 + t^5/5 - ... to t^17/17 (truncation < 8e-13). */
BSX_HD float bsx_atan_unit(float t) {
    const float kTanPi12 = 0.2679491937160492f;
    const float kInvSqrt3 = 0.5773502588272095f;
    const float kPi6Hi = 0.5235987901687622f;     /* float(pi/6) */
    const float kPi6Lo = -2.2841566377645488e-08f; /* pi/6 - kPi6Hi */
    int reduced = t > kTanPi12;
    float x = reduced ? (t - kInvSqrt3) / bsx_fma(t, kInvSqrt3, 1.0f) : t;
    float x2 = x * x;
    float p = 0.05882352963089943f;             /* 1/17 */
    p = bsx_fma(p, x2, -0.06666667014360428f);  /* -1/15 */
    p = bsx_fma(p, x2, 0.07692307978868484f);   /* 1/13 */
    p = bsx_fma(p, x2, -0.09090909361839294f);  /* -1/11 */
    p = bsx_fma(p, x2, 0.1111111119389534f);    /* 1/9 */
    p = bsx_fma(p, x2, -0.1428571492433548f);   /* -1/7 */
    p = bsx_fma(p, x2, 0.20000000298023224f);   /* 1/5 */
    p = bsx_fma(p, x2, -0.3333333432674408f);   /* -1/3 */
    float r = bsx_fma(x * x2, p, x);
    return reduced ? (kPi6Hi + (r + kPi6Lo)) : r;
}

/* atan2(y, x) in float32 with the C library's quadrant and special-value
 * conventions: the ratio of the smaller to the larger magnitude goes through
 * bsx_atan_unit, then pi/2 - r, pi - r and the sign of y place it. */
BSX_HD float bsx_atan2f(float y, float x) {
    const float kPi2Hi = 1.5707963705062866f, kPi2Lo = -4.371139000186243e-08f;
    const float kPiHi = 3.1415927410125732f, kPiLo = -8.742278000372485e-08f;
    if (x != x || y != y) return x + y;
    float ax = x < 0.0f ? -x : x, ay = y < 0.0f ? -y : y;
    int neg_x = (bsx_f32_to_bits(x) >> 31) != 0;
    int neg_y = (bsx_f32_to_bits(y) >> 31) != 0;
    float r;
    if (ay == 0.0f) {
        r = neg_x ? kPiHi : 0.0f;
    } else if (ax == bsx_bits_to_f32(0x7f800000u) && ay == ax) {
        r = neg_x ? 2.356194496154785f : 0.7853981852531433f; /* 3pi/4, pi/4 */
    } else if (ax == bsx_bits_to_f32(0x7f800000u)) {
        r = neg_x ? kPiHi : 0.0f;
    } else if (ay == bsx_bits_to_f32(0x7f800000u) || ax == 0.0f) {
        r = kPi2Hi;
    } else {
        int swap = ay > ax;
        float t = swap ? ax / ay : ay / ax;
        r = bsx_atan_unit(t);
        if (swap) r = kPi2Hi + (kPi2Lo - r);
        if (neg_x) r = kPiHi + (kPiLo - r);
    }
    return neg_y ? -r : r;
}

/* Logistic sigmoid, same expression as the reference: 1 / (1 + e^-x). */
BSX_HD float bsx_sigmoid(float x) { return 1.0f / (1.0f + bsx_expf(-x)); }

/* b^e for an integer exponent by binary exponentiation (square-and-multiply,
 * least significant bit first): a fixed operation sequence for every e. */
BSX_HD float bsx_powi(float b, uint32_t e) {
    float r = 1.0f;
    while (e) {
        if (e & 1u) r = r * b;
        e >>= 1;
        if (e) b = b * b;
    }
    return r;
}

/* SplitMix64 (Steele, Lea, Flood 2014): a 64-bit counter hash. */
BSX_HD uint64_t bsx_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* sin(2 pi u) and cos(2 pi u) for u in [0, 1). The turn is split into eighths
 * exactly (8u, its integer part q and fraction f are exact in float); an odd
 * eighth is mirrored (f -> 1 - f, exact), so the remaining angle a = f pi/4 lies
 * in [0, pi/4], where the Maclaurin series of sin to a^11 and cos to a^12 are
 * within 2e-11 of the exact values; the eighth then selects sign and
 * sin / cos swap. */
BSX_HD void bsx_sincos_2pi(float u, float* s, float* c) {
    const float y = u * 8.0f;
    const int q = (int)y;
    float f = y - (float)q;
    if (q & 1) f = 1.0f - f;
    const float a = f * 0.7853981852531433f; /* pi/4 */
    const float a2 = a * a;
    float ps = -2.505210838544172e-08f;          /* -1/11! */
    ps = bsx_fma(ps, a2, 2.755731922398589e-06f); /* 1/9! */
    ps = bsx_fma(ps, a2, -1.9841270114481449e-04f); /* -1/7! */
    ps = bsx_fma(ps, a2, 8.333333767950535e-03f);  /* 1/5! */
    ps = bsx_fma(ps, a2, -0.1666666716337204f);    /* -1/3! */
    const float sa = bsx_fma(a * a2, ps, a);
    float pc = 2.08767569878681e-09f;              /* 1/12! */
    pc = bsx_fma(pc, a2, -2.755731922398589e-07f); /* -1/10! */
    pc = bsx_fma(pc, a2, 2.4801587642286904e-05f); /* 1/8! */
    pc = bsx_fma(pc, a2, -1.3888889225199819e-03f); /* -1/6! */
    pc = bsx_fma(pc, a2, 0.0416666679084301f);     /* 1/4! */
    pc = bsx_fma(pc, a2, -0.5f);
    const float ca = bsx_fma(a2, pc, 1.0f);
    /* within the quadrant: even eighth -> (sin a, cos a); odd -> (cos a', sin a') */
    const float sq = (q & 1) ? ca : sa, cq = (q & 1) ? sa : ca;
    switch ((q >> 1) & 3) {
        case 0: *s = sq; *c = cq; break;
        case 1: *s = cq; *c = -sq; break;
        case 2: *s = -sq; *c = -cq; break;
        default: *s = -cq; *c = sq; break;
    }
}

/* Three standard normal variates for (seed, step, splat index), by the
 * Box-Muller transform of two counter-hashed uniform pairs
 * (u1 in (0, 1], u2 in [0, 1), 24 bits each): r = sqrt(-2 ln u1),
 * (r cos 2 pi u2, r sin 2 pi u2). Deterministic and identical on the host and
 * the device. */
BSX_HD void bsx_normal3(uint64_t seed, uint32_t step, uint32_t index, float z[3]) {
    const uint64_t base = bsx_splitmix64(seed ^ ((uint64_t)step << 32));
    for (int pair = 0; pair < 2; ++pair) {
        const uint64_t h = bsx_splitmix64(base ^ bsx_splitmix64(((uint64_t)index << 1) | (uint64_t)pair));
        const float u1 = (float)((h >> 40) + 1) * 5.9604644775390625e-08f;         /* (0, 1] */
        const float u2 = (float)((h >> 16) & 0xFFFFFFull) * 5.9604644775390625e-08f; /* [0, 1) */
        const float r = sqrtf(-2.0f * bsx_logf(u1));
        float sn, cs;
        bsx_sincos_2pi(u2, &sn, &cs);
        if (pair == 0) {
            z[0] = r * cs;
            z[1] = r * sn;
        } else {
            z[2] = r * cs;
        }
    }
}

/* The mean-noise step of one splat (crates/brush-train/src/train.rs:1095-1169):
 * w = clamp((1 - sigmoid(raw_opac))^150, 0, 1) * gate, gate in {0, 1};
 * each mean coordinate moves by clamp(n_k * (w * scale), -limit, limit), with
 * scale = f32(lr_mean) * mean_noise_weight and limit = the median bounds size.
 * Returns 0 (means unchanged) where the weight is zero. */
BSX_HD int bsx_mean_noise(float raw_opac, float gate, float scale, float limit, uint64_t seed, uint32_t step,
                          uint32_t index, float mean[3]) {
    const float inv = 1.0f - bsx_sigmoid(raw_opac);
    const float w = bsx_clamp(bsx_powi(inv, 150u), 0.0f, 1.0f) * gate;
    if (!(w != 0.0f)) return 0;
    const float wm = w * scale;
    /* Exact shortcut: |n| <= sqrt(-2 ln 2^-24) < 5.77 for these uniforms, so each
     * move is at most 5.78 |wm|. Below 2^(e-25) for a finite mean in [2^e, 2^(e+1))
     * (half the float spacing on either side) the rounded sum is the mean itself,
     * and the normals need not be drawn. */
    {
        int noop = 1;
        const float bound = 5.78f * (wm < 0.0f ? -wm : wm);
        for (int k = 0; k < 3 && noop; ++k) {
            const uint32_t e = (bsx_f32_to_bits(mean[k]) >> 23) & 0xFFu;
            noop = e != 0xFFu && e >= 26u && bound < bsx_bits_to_f32((e - 25u) << 23);
        }
        if (noop) return 0;
    }
    float z[3];
    bsx_normal3(seed, step, index, z);
    for (int k = 0; k < 3; ++k) mean[k] = mean[k] + bsx_clamp(z[k] * wm, -limit, limit);
    return 1;
}

#endif /* BSX_FMATH_H */
