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
// The reference calls glibc expf / log1pf there. Their results differ from the correctly
// rounded ones by one ulp for a small fraction of inputs, and any such difference changes the
// greedy tokens downstream (the int8 activation quantisation amplifies it), so the device
// reproduces glibc's values: the correctly rounded result, computed in double precision,
// corrected by a per-input 2-bit code from a table that the host builds by calling glibc's
// own expf / log1pf on every input of the domain (nb_libm.cpp). Code 3 marks inputs whose
// double result lies so close to a float rounding boundary that a different double
// implementation could round it the other way; their glibc values are in a small sorted list.
struct LibmTables {
    const uint32_t *exp_bits;    // 2-bit codes, inputs |x| in [kLo, kExpHiBits], both signs
    const uint32_t *log1p_bits;  // 2-bit codes, inputs y in [kLo, kLog1pHiBits]
    const uint32_t *ovf_key;     // sorted (function << 32 | input bits) of code-3 inputs
    const float *ovf_val;
    int n_ovf;
};
constexpr uint32_t kLibmLo = 0x30800000u;        // 2^-30
constexpr uint32_t kExpHiBits = 0x42D00000u;     // 104.0
constexpr uint32_t kLog1pHiBits = 0x4DE80000u;   // 4.866e8 > expf(20)
constexpr uint32_t kExpSpan = kExpHiBits - kLibmLo + 1;


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

__device__ __forceinline__ uint32_t libm_code(const uint32_t *t, uint32_t idx) {
    return (__ldg(t + (idx >> 4)) >> ((idx & 15u) * 2u)) & 3u;
}

static __device__ __noinline__ float libm_overflow(const LibmTables &L, uint32_t fn, uint32_t bits,
                                            float fallback) {
    const uint64_t key = ((uint64_t)fn << 32) | bits;
    int lo = 0, hi = L.n_ovf - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        const uint64_t k = ((uint64_t)L.ovf_key[2 * mid] << 32) | L.ovf_key[2 * mid + 1];
        if (k == key) return L.ovf_val[mid];
        if (k < key) lo = mid + 1; else hi = mid - 1;
    }
    return fallback;
}

__device__ __forceinline__ float apply_code(uint32_t code, float c) {
    const uint32_t cb = __float_as_uint(c);
    return code == 1u ? __uint_as_float(cb + 1u) : (code == 2u ? __uint_as_float(cb - 1u) : c);
}

// glibc expf(x)
__device__ __forceinline__ float glibc_expf(const LibmTables &L, float x) {
    const float c = __double2float_rn(exp((double)x));
    const uint32_t b = __float_as_uint(x), a = b & 0x7fffffffu;
    if (a < kLibmLo || a > kExpHiBits) return c;
    const uint32_t idx = (b >> 31) * kExpSpan + (a - kLibmLo);
    const uint32_t code = libm_code(L.exp_bits, idx);
    if (code == 3u) return libm_overflow(L, 0u, b, c);
    return apply_code(code, c);
}

// glibc log1pf(y) for y >= 0 (the only inputs the reference passes: y = expf(x))
__device__ __forceinline__ float glibc_log1pf(const LibmTables &L, float y) {
    const float c = __double2float_rn(log1p((double)y));
    const uint32_t b = __float_as_uint(y);
    if (b < kLibmLo || b > kLog1pHiBits) return c;
    const uint32_t code = libm_code(L.log1p_bits, b - kLibmLo);
    if (code == 3u) return libm_overflow(L, 1u, b, c);
    return apply_code(code, c);
}

#endif  // __CUDACC__

}  // namespace nb
