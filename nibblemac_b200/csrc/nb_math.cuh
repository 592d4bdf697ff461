// Device restatements of the reference engine's scalar float primitives, bit for bit.
//
// The reference's forward pass is fp32 with a fixed operation order and no fused
// multiply-add (engine/src/forward_ops.c:1-14, built with -ffp-contract=off); its NEON and
// scalar bodies agree bit for bit, so matching the scalar mirror matches the reference on
// every host. Every helper here spells each rounding step with an IEEE intrinsic
// (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn), which nvcc never contracts or reorders, so
// the results do not depend on --fmad or fast-math flags. The only fused steps are the ones
// the reference fuses explicitly (the Q4K block FMAs, written with __fmaf_rn where used).
#pragma once
#include <cstdint>

namespace nb {

// ---- libm scalars of the DeltaNet gates (engine/src/forward_lin.c:19,290-293) ----------
// The reference calls the host C library's expf and log1pf there, and the greedy tokens depend
// on their last bits (the int8 activation quantisation amplifies a one-ulp change). glibc's
// results are not the correctly rounded ones (they differ for ~0.03% of expf inputs and ~1.5%
// of log1pf inputs), so the device evaluates glibc's own published algorithms, restated below
// with every rounding step explicit. The same source compiles for the host, where
// nb_libm_selftest compares it with the C library input by input (all 2^32 inputs when asked:
// identical on glibc 2.39, x86-64 with FMA).
//   glibc_expf: the exp2f-table method of glibc's expf (sysdeps/ieee754/flt-32/e_expf.c):
//     k = round(x * 32 / ln 2), r = x * 32 / ln 2 - k (both by fused multiply-add, as glibc's
//     FMA build computes them), 2^(k/32) from a 32-entry table of 2^(i/32) plus the exponent
//     bits, and a cubic in r, all in double precision, rounded to float once at the end.
//   glibc_log1pf: the fdlibm single-precision log1p (sysdeps/ieee754/flt-32/s_log1pf.c):
//     argument reduction 1 + x = 2^k (1 + f) with a correction term for the rounding of 1 + x,
//     s = f / (2 + f), a degree-7 polynomial in s^2, and k ln 2 in two parts; float arithmetic.
#if defined(__CUDACC__)
#define NB_HD __host__ __device__ __forceinline__
#else
#define NB_HD inline
#endif
#if defined(__CUDA_ARCH__)
#define NB_FMUL(a, b) __fmul_rn((a), (b))
#define NB_FADD(a, b) __fadd_rn((a), (b))
#define NB_FSUB(a, b) __fsub_rn((a), (b))
#define NB_FDIV(a, b) __fdiv_rn((a), (b))
#define NB_DMUL(a, b) __dmul_rn((a), (b))
#define NB_DSUB(a, b) __dsub_rn((a), (b))
#define NB_DFMA(a, b, c) __fma_rn((a), (b), (c))
#define NB_D2F(a) __double2float_rn(a)
#else
#define NB_FMUL(a, b) ((a) * (b))
#define NB_FADD(a, b) ((a) + (b))
#define NB_FSUB(a, b) ((a) - (b))
#define NB_FDIV(a, b) ((a) / (b))
#define NB_DMUL(a, b) ((a) * (b))
#define NB_DSUB(a, b) ((a) - (b))
#define NB_DFMA(a, b, c) __builtin_fma((a), (b), (c))
#define NB_D2F(a) ((float)(a))
#endif

NB_HD uint32_t libm_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
    return u;
#endif
}
NB_HD float libm_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}
NB_HD uint64_t libm_d2u(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u;
    __builtin_memcpy(&u, &d, 8);
    return u;
#endif
}
NB_HD double libm_u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d;
    __builtin_memcpy(&d, &u, 8);
    return d;
#endif
}

// Order-preserving key of a (logit, row) pair: larger logit wins, then the lower row, NaN never
// wins (pf_argmax, engine/src/forward_ops.c:387-409: first maximum, NaN skipped); the maximum
// over any split of the rows (panels, warps, vocab shards) is the maximum over all of them.
NB_HD unsigned long long argmax_key(float v, int row) {
    uint32_t u = libm_f2u(v);
    if (v != v) u = 0u;
    else if (v == 0.0f) u = 0x80000000u;                 // +0 and -0 compare equal
    else u = (u >> 31) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xffffffffu - (uint32_t)row);
}

// bits of 2^(i/32) rounded to the nearest double, minus i << 47 (so that adding k << 47 for
// k = 32 m + i gives 2^(k/32) directly)
#define NB_EXP2_TAB {                                                             \
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL, \
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL, \
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL, \
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL, \
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL, \
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL, \
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL, \
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL }
#if defined(__CUDACC__)
static __constant__ uint64_t kExp2TabDev[32] = NB_EXP2_TAB;
#endif
static const uint64_t kExp2TabHost[32] = NB_EXP2_TAB;

NB_HD float glibc_expf(float x) {
    const double kInvLn2N = 0x1.71547652b82fep+0 * 32;   // 32 / ln 2
    const double kShift = 0x1.8p+52;                      // round-to-integer by addition
    const double kC0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double kC1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const uint32_t b = libm_f2u(x), top = (b >> 20) & 0x7ffu;
    if (top >= 0x42bu) {                       // |x| >= 88, inf or nan
        if (b == 0xff800000u) return 0.0f;     // exp(-inf)
        if (top >= 0x7f8u) return NB_FADD(x, x);
        if (x > 0x1.62e42ep6f) return libm_u2f(0x7f800000u);   // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;                   // underflow below 2^-150
    }
    const double xd = (double)x;
    double kd = NB_DFMA(kInvLn2N, xd, kShift);
    const uint64_t ki = libm_d2u(kd);
    kd = NB_DSUB(kd, kShift);
    const double r = NB_DFMA(kInvLn2N, xd, -kd);
#if defined(__CUDA_ARCH__)
    uint64_t t = kExp2TabDev[ki % 32];
#else
    uint64_t t = kExp2TabHost[ki % 32];
#endif
    t += ki << 47;
    const double s = libm_u2d(t);
    const double z = NB_DFMA(kC0, r, kC1);
    const double r2 = NB_DMUL(r, r);
    double y = NB_DFMA(kC2, r, 1.0);
    y = NB_DFMA(z, r2, y);
    y = NB_DMUL(y, s);
    return NB_D2F(y);
}

NB_HD float glibc_log1pf(float x) {
    const float ln2_hi = libm_u2f(0x3f317180u), ln2_lo = libm_u2f(0x3717f7d1u);
    const float P1 = libm_u2f(0x3f2aaaabu), P2 = libm_u2f(0x3ecccccdu), P3 = libm_u2f(0x3e924925u),
                P4 = libm_u2f(0x3e638e29u), P5 = libm_u2f(0x3e3a3325u), P6 = libm_u2f(0x3e1cd04fu),
                P7 = libm_u2f(0x3e178897u);
    const int32_t hx = (int32_t)libm_f2u(x), ax = hx & 0x7fffffff;
    int k = 1, hu = 0;
    float f = 0.0f, c = 0.0f;
    if (hx < 0x3ed413d7) {                                  // x < 0.41422 (or negative)
        if (ax >= 0x3f800000)                               // x <= -1
            return x == -1.0f ? libm_u2f(0xff800000u) : libm_u2f(0x7fc00000u);
        if (ax < 0x31000000) {                              // |x| < 2^-29
            if (ax < 0x24800000) return x;                  // |x| < 2^-54
            return NB_FSUB(x, NB_FMUL(NB_FMUL(x, x), 0.5f));
        }
        if (hx > 0 || hx <= (int32_t)0xbe95f61fu) {         // -0.2929 < x < 0.41422: f = x
            k = 0;
            f = x;
            hu = 1;
        }
    } else if (hx >= 0x7f800000) {
        return NB_FADD(x, x);
    }
    if (k != 0) {
        float u;
        if (hx < 0x5a000000) {
            u = NB_FADD(1.0f, x);
            hu = (int32_t)libm_f2u(u);
            k = (hu >> 23) - 127;
            c = k > 0 ? NB_FSUB(1.0f, NB_FSUB(u, x)) : NB_FSUB(x, NB_FSUB(u, 1.0f));   // rounding of 1 + x
            c = NB_FDIV(c, u);
        } else {
            u = x;
            hu = (int32_t)libm_f2u(u);
            k = (hu >> 23) - 127;
            c = 0.0f;
        }
        hu &= 0x007fffff;
        if (hu < 0x3504f7) {
            u = libm_u2f((uint32_t)hu | 0x3f800000u);      // u in [1, sqrt 2)
        } else {
            k += 1;
            u = libm_u2f((uint32_t)hu | 0x3f000000u);      // u / 2
            hu = (0x00800000 - hu) >> 2;
        }
        f = NB_FSUB(u, 1.0f);
    }
    const float hfsq = NB_FMUL(NB_FMUL(0.5f, f), f);
    const float kf = (float)k;
    if (hu == 0) {                                          // |f| < 2^-20
        if (f == 0.0f) {
            if (k == 0) return 0.0f;
            c = NB_FADD(c, NB_FMUL(kf, ln2_lo));
            return NB_FADD(NB_FMUL(kf, ln2_hi), c);
        }
        const float R = NB_FMUL(hfsq, NB_FSUB(1.0f, NB_FMUL(libm_u2f(0x3f2aaaabu), f)));
        if (k == 0) return NB_FSUB(f, R);
        return NB_FSUB(NB_FMUL(kf, ln2_hi), NB_FSUB(NB_FSUB(R, NB_FADD(NB_FMUL(kf, ln2_lo), c)), f));
    }
    const float s = NB_FDIV(f, NB_FADD(2.0f, f));
    const float z = NB_FMUL(s, s);
    float R = NB_FMUL(z, P7);
    R = NB_FMUL(z, NB_FADD(P6, R));
    R = NB_FMUL(z, NB_FADD(P5, R));
    R = NB_FMUL(z, NB_FADD(P4, R));
    R = NB_FMUL(z, NB_FADD(P3, R));
    R = NB_FMUL(z, NB_FADD(P2, R));
    R = NB_FMUL(z, NB_FADD(P1, R));
    const float t = NB_FMUL(s, NB_FADD(hfsq, R));
    if (k == 0) return NB_FSUB(f, NB_FSUB(hfsq, t));
    return NB_FSUB(NB_FMUL(kf, ln2_hi), NB_FSUB(NB_FSUB(hfsq, NB_FADD(t, NB_FADD(NB_FMUL(kf, ln2_lo), c))), f));
}

#if defined(__CUDACC__)

// Reference constants of pf_expf (engine/src/forward_ops.c:28-39): clamp range, log2(e), ln 2
// split in two parts, degree-6 polynomial coefficients.
constexpr float kExpHi = 88.0f;
constexpr float kExpLo = -87.0f;
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693145751953125f;
constexpr float kLn2Lo = 1.428606765330187e-06f;
constexpr float kEp0 = 1.9875691500e-4f;
constexpr float kEp1 = 1.3981999507e-3f;
constexpr float kEp2 = 8.3334519073e-3f;
constexpr float kEp3 = 4.1665795894e-2f;
constexpr float kEp4 = 1.6666665459e-1f;
constexpr float kEp5 = 5.0000001201e-1f;

// pf_expf (forward_ops.c:41-56): clamp, n = rint(x log2 e), r = x - n ln2 in two steps,
// y = p(r) r^2 + r + 1, times 2^n assembled from the exponent bits.
__device__ __forceinline__ float pf_expf(float x) {
    x = x < kExpLo ? kExpLo : (x > kExpHi ? kExpHi : x);
    const float fx = rintf(__fmul_rn(x, kLog2e));
    float r = __fadd_rn(x, -__fmul_rn(fx, kLn2Hi));
    r = __fadd_rn(r, -__fmul_rn(fx, kLn2Lo));
    float p = kEp0;
    p = __fadd_rn(__fmul_rn(p, r), kEp1);
    p = __fadd_rn(__fmul_rn(p, r), kEp2);
    p = __fadd_rn(__fmul_rn(p, r), kEp3);
    p = __fadd_rn(__fmul_rn(p, r), kEp4);
    p = __fadd_rn(__fmul_rn(p, r), kEp5);
    float y = __fadd_rn(__fmul_rn(p, __fmul_rn(r, r)), r);
    y = __fadd_rn(y, 1.0f);
    const float s = __uint_as_float((uint32_t)((int)fx + 127) << 23);
    return __fmul_rn(y, s);
}

// pf_silu / pf_sigmoid (forward_ops.c:58-59)
__device__ __forceinline__ float pf_silu(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, pf_expf(-x)));
}
__device__ __forceinline__ float pf_sigmoid(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, pf_expf(-x)));
}

// a * b with separate rounding, then + c (the reference's "acc = acc + a * b")
__device__ __forceinline__ float madd(float acc, float a, float b) {
    return __fadd_rn(acc, __fmul_rn(a, b));
}

// 1 / sqrt(v) as the reference writes it: 1.0f / sqrtf(v), both correctly rounded.
__device__ __forceinline__ float inv_sqrt_ref(float v) {
    return __fdiv_rn(1.0f, __fsqrt_rn(v));
}

#endif  // __CUDACC__

}  // namespace nb
