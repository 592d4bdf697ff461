// Device helpers shared by the kernel sources (nb_kernels.cu, nb_gemm.cu): programmatic
// dependent launch, warp reductions, the A8 block quantiser, and the mbarrier / bulk-copy PTX.
// Everything is in an anonymous namespace: each translation unit gets its own copy.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>
#include <utility>

#include "nb_engine.h"

namespace nb {
namespace {

// ------------------------------------------------------------------ programmatic dependent launch
// Every kernel of the forward is launched with programmatic stream serialisation, so it can be
// resident while its predecessor on the stream finishes. Each kernel calls pdl_wait() before it
// touches anything another kernel writes (griddepcontrol.wait returns once every prerequisite
// grid has completed and its memory is visible) and only then pdl_trigger(), which lets the
// next kernel launch. Hence, while a kernel runs code placed before its pdl_wait(), every kernel
// earlier than its immediate predecessor has completed, and that code reads only data the
// predecessor does not write (weights, and state the predecessor never touches).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <class... KArgs, class... Args>
void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ warp helpers
__device__ __forceinline__ float warp_max_abs(float v) {
    float m = fabsf(v);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}
__device__ __forceinline__ int warp_sum_int(int v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
    for (int o = 16; o; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// A8 quantisation of one 32-column block held one value per lane (kern_quant_act,
// engine/src/kern_act.c:14-41): amax = max |x|, id = amax > 0 ? 127 / amax : 0,
// q = round-half-even(x * id) (vcvtnq: NaN -> 0, saturating), d = amax / 127,
// fsum = d * (float)sum(q). Writes q at qdst[lane] and d / fsum through lane 0.
__device__ __forceinline__ void quant_block_warp(float x, int lane, int8_t *qdst, float *ddst,
                                                 float *fdst) {
    const float amax = warp_max_abs(x);
    const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    const int q = __float2int_rn(__fmul_rn(x, id));
    const int sum = warp_sum_int(q);
    qdst[lane] = (int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
    if (lane == 0) {
        const float d = __fdiv_rn(amax, 127.0f);
        *ddst = d;
        *fdst = __fmul_rn(d, (float)sum);
    }
}

// The same A8 of one 32-column block held by a group of 8 lanes, 4 consecutive columns per lane
// (sub = lane & 7): max, division, rounding and code sum are order-independent, so the bits
// match quant_block_warp. Four blocks per warp at a time, 3-step shuffles; every lane of the
// warp must call it. qdst: the block's 32 codes; lane sub writes bytes 4 sub .. 4 sub + 3 and
// sub 0 writes d and fsum, unless store is false (a padding group).
__device__ __forceinline__ void quant_block_oct(const float (&x)[4], int sub, bool store, int8_t *qdst,
                                                float *ddst, float *fdst) {
    float a = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
    const float id = a > 0.0f ? __fdiv_rn(127.0f, a) : 0.0f;
    int sum = 0;
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = __float2int_rn(__fmul_rn(x[i], id));
        sum += q;
        packed |= (uint32_t)(uint8_t)(int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q)) << (8 * i);
    }
    if (store) *reinterpret_cast<uint32_t *>(qdst + 4 * sub) = packed;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (store && sub == 0) {
        const float d = __fdiv_rn(a, 127.0f);
        *ddst = d;
        *fdst = __fmul_rn(d, (float)sum);
    }
}


__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    return __half2float(__ushort_as_half((unsigned short)h));
}


// ------------------------------------------------------------------ mbarriers and bulk copies
constexpr unsigned kSpinLimit = 1u << 22;   // bounded mbarrier waits

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// expect `bytes` and start the bulk copy global -> shared that completes them
__device__ __forceinline__ void tma_load_1d(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// one arrival that also announces `bytes` of bulk copies still to complete on the barrier
__device__ __forceinline__ void mbar_arrive_expect(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// bulk copy global -> shared completing on `bar` (no arrival of its own)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// wait for phase `parity` of the barrier; false after `limit` polls (the caller reports
// the timeout instead of hanging)
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned limit = kSpinLimit) {
    const uint32_t a = smem_u32(bar);
    for (unsigned i = 0; i < limit; i++) {
        uint32_t ok;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(a), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}

__device__ __forceinline__ uint4 lds128(const uint8_t *p) {
    return *reinterpret_cast<const uint4 *>(p);
}

}  // namespace
}  // namespace nb
