// Device kernels of the B200 verify path (sm_100a).
//
// Every kernel reproduces the reference engine's arithmetic bit for bit (file:line cited per
// kernel); nb_math.cuh holds the shared scalar primitives. Kernels read the pass shape (rows n,
// first position pos0, logged or not) from the Step block in device memory, so one captured
// CUDA graph serves every round of a generation.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <utility>
#include <cstdio>

#include "nb_dev.cuh"
#include "nb_engine.h"

namespace nb {

namespace {

__device__ __forceinline__ int dot_block(const uint4 c, const int4 x0, const int4 x1) {
    // 16 code bytes: byte j = column j (low nibble) | column j + 16 (high nibble)
    int s = 0;
    s = __dp4a((int)(c.x & 0x0f0f0f0fu), x0.x, s);
    s = __dp4a((int)(c.y & 0x0f0f0f0fu), x0.y, s);
    s = __dp4a((int)(c.z & 0x0f0f0f0fu), x0.z, s);
    s = __dp4a((int)(c.w & 0x0f0f0f0fu), x0.w, s);
    s = __dp4a((int)((c.x >> 4) & 0x0f0f0f0fu), x1.x, s);
    s = __dp4a((int)((c.y >> 4) & 0x0f0f0f0fu), x1.y, s);
    s = __dp4a((int)((c.z >> 4) & 0x0f0f0f0fu), x1.z, s);
    s = __dp4a((int)((c.w >> 4) & 0x0f0f0f0fu), x1.w, s);
    return s;
}

// ------------------------------------------------------------------ Q4K x A8 matvec
// Per (row, vector) the reference computes, blocks in column order (kern_q4k / q4_tile /
// q4_block, engine/src/kern_quant.c:148-245):
//   isum = sum_j u[j] * q[j]                     (int32, exact)
//   acc  = fmaf((float)isum, (D * s6) * d_act, acc)
//   acc  = fmaf(-(M * m6), fsum_act, acc)
// A CTA of 4 warps owns one 32-row panel (lane = row). The superblocks of the row are split
// over the warps in chunks of 4: each warp computes the integer block dots of one superblock
// (coalesced 512-byte loads, dp4a on CUDA cores), then the ordered FMA chain runs over the
// chunk's 32 blocks from shared memory, one thread per (row, vector). The chain order, and so
// every bit of the result, is independent of n and of the split.
constexpr int kMvWarps = 4;
constexpr int kMvThreads = kMvWarps * 32;

template <int NMAX>
struct MvSmem {
    int32_t isum[kMvWarps * 8][NMAX][32];
    float ds[kMvWarps * 8][32];
    float os[kMvWarps * 8][32];
    float da[NMAX][kMvWarps * 8];
    float fa[NMAX][kMvWarps * 8];
};

template <int NMAX>
__device__ __forceinline__ void mv_panel(const Mat &W, const Act &in, int n, int panel,
                                         MvSmem<NMAX> &sm, float (&acc)[(NMAX + 3) / 4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = W.cols >> 5;
#pragma unroll
    for (int i = 0; i < (NMAX + 3) / 4; i++) acc[i] = 0.0f;
    for (int c0 = 0; c0 < W.nsb; c0 += kMvWarps) {
        const int sb = c0 + warp;
        if (sb < W.nsb) {
            const uint8_t *u = W.w + ((size_t)panel * W.nsb + sb) * kUnitBytes + lane * 16;
            const uint4 sc = __ldcs(reinterpret_cast<const uint4 *>(u));
            uint4 cd[8];
#pragma unroll
            for (int k = 0; k < 8; k++) cd[k] = __ldcs(reinterpret_cast<const uint4 *>(u + 512 * (k + 1)));
            const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
            const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
            const float D = half_bits_to_float((uint32_t)(A >> 48));
            const float M = half_bits_to_float((uint32_t)(B >> 48));
#pragma unroll
            for (int k = 0; k < 8; k++) {
                sm.ds[warp * 8 + k][lane] = __fmul_rn(D, (float)(uint32_t)((A >> (6 * k)) & 63u));
                sm.os[warp * 8 + k][lane] = __fmul_rn(M, (float)(uint32_t)((B >> (6 * k)) & 63u));
            }
            for (int v = 0; v < n; v++) {
                const int4 *xq = reinterpret_cast<const int4 *>(in.q + (size_t)v * in.cols + sb * 256);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int4 x0 = __ldg(xq + 2 * k), x1 = __ldg(xq + 2 * k + 1);
                    sm.isum[warp * 8 + k][v][lane] = dot_block(cd[k], x0, x1);
                }
                if (lane < 8) {
                    sm.da[v][warp * 8 + lane] = __ldg(in.d + (size_t)v * nb + sb * 8 + lane);
                    sm.fa[v][warp * 8 + lane] = __ldg(in.fs + (size_t)v * nb + sb * 8 + lane);
                }
            }
        }
        __syncthreads();
        const int left = W.nsb - c0;
        const int nblk = (left < kMvWarps ? left : kMvWarps) * 8;
#pragma unroll
        for (int i = 0; i < (NMAX + 3) / 4; i++) {
            const int v = warp + 4 * i;
            if (v < n) {
                float a = acc[i];
                for (int b = 0; b < nblk; b++) {
                    const float s = (float)sm.isum[b][v][lane];
                    a = __fmaf_rn(s, __fmul_rn(sm.ds[b][lane], sm.da[v][b]), a);
                    a = __fmaf_rn(-sm.os[b][lane], sm.fa[v][b], a);
                }
                acc[i] = a;
            }
        }
        __syncthreads();
    }
}

// mode 0: y[v][row] = acc; mode 1: y[v][row] += acc (residual, pf_add_rows
// engine/src/forward.c:68-72: x = x + out)
template <int NMAX, int MODE>
__global__ void __launch_bounds__(kMvThreads) k_matvec(Mat W, Act in, const Step *st, float *y,
                                                       int ldy) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smraw[];
    MvSmem<NMAX> &sm = *reinterpret_cast<MvSmem<NMAX> *>(smraw);
    const int n = st->n;
    if (n <= 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int panel = blockIdx.x; panel < W.npanels; panel += gridDim.x) {
        float acc[(NMAX + 3) / 4];
        mv_panel<NMAX>(W, in, n, panel, sm, acc);
        const int row = panel * kPanelRows + lane;
#pragma unroll
        for (int i = 0; i < (NMAX + 3) / 4; i++) {
            const int v = warp + 4 * i;
            if (v < n && row < W.rows) {
                float *p = y + (size_t)v * ldy + row;
                *p = MODE == 0 ? acc[i] : __fadd_rn(*p, acc[i]);
            }
        }
    }
}

// Tied LM head (engine/src/forward.c:142-145): logits of every row and, per panel, the
// (max, first index) key of every vector for the on-device argmax.
template <int NMAX>
__global__ void __launch_bounds__(kMvThreads) k_matvec_head(Mat W, Act in, const Step *st,
                                                            float *logits, int ld,
                                                            unsigned long long *partial,
                                                            int *nan0) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smraw[];
    MvSmem<NMAX> &sm = *reinterpret_cast<MvSmem<NMAX> *>(smraw);
    const int n = st->n;
    if (n <= 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int panel = blockIdx.x; panel < W.npanels; panel += gridDim.x) {
        float acc[(NMAX + 3) / 4];
        mv_panel<NMAX>(W, in, n, panel, sm, acc);
        const int row = panel * kPanelRows + lane;
#pragma unroll
        for (int i = 0; i < (NMAX + 3) / 4; i++) {
            const int v = warp + 4 * i;
            if (v < n) {   // warp-uniform
                if (logits && row < W.rows) logits[(size_t)v * ld + row] = acc[i];
                const unsigned long long key = row < W.rows ? argmax_key(acc[i], row) : 0ull;
                const unsigned long long best = warp_max_u64(key);
                if (lane == 0) partial[(size_t)v * W.npanels + panel] = best;
                if (panel == 0 && lane == 0) nan0[v] = acc[i] != acc[i];
            }
        }
    }
}

// gate / up projections with SwiGLU (pf_mlp + pf_silu_mul, engine/src/forward.c:49-58,
// forward_ops.c:98-101: h = silu(g) * u) and the A8 quantisation of h for the down projection
// (one 32-row panel = one 32-column activation block).
template <int NMAX>
__global__ void __launch_bounds__(kMvThreads) k_matvec_swiglu(Mat G, Mat U, Act in,
                                                              const Step *st, Act out) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smraw[];
    MvSmem<NMAX> &sm = *reinterpret_cast<MvSmem<NMAX> *>(smraw);
    const int n = st->n;
    if (n <= 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nbo = out.cols >> 5;
    for (int panel = blockIdx.x; panel < G.npanels; panel += gridDim.x) {
        float g[(NMAX + 3) / 4], u[(NMAX + 3) / 4];
        mv_panel<NMAX>(G, in, n, panel, sm, g);
        mv_panel<NMAX>(U, in, n, panel, sm, u);
#pragma unroll
        for (int i = 0; i < (NMAX + 3) / 4; i++) {
            const int v = warp + 4 * i;
            if (v < n) {
                const float h = __fmul_rn(pf_silu(g[i]), u[i]);
                quant_block_warp(h, lane, out.q + (size_t)v * out.cols + panel * 32,
                                 out.d + (size_t)v * nbo + panel, out.fs + (size_t)v * nbo + panel);
            }
        }
    }
}

// ------------------------------------------------------------------ TMA-fed matvec
// The same per-(row, vector) arithmetic as mv_panel, restructured for HBM streaming on B200:
// weight units (one 32-row panel x 256 columns, 4608 bytes) are fetched with cp.async.bulk
// (TMA bulk copies, completion counted on an mbarrier) into a ring of shared-memory slots per
// warp, so every SM keeps ~110 KB of weights in flight while its warps compute. A warp owns
// whole panels (lane = row) and walks their superblocks in column order, so the ordered FMA
// chain of every (row, vector) stays in registers and never crosses warps.
constexpr int kTallWarps = 8;
constexpr int kRing = 2;
constexpr size_t kTallSmem = (size_t)kTallWarps * kRing * kUnitBytes + kTallWarps * kRing * 8;
__device__ __forceinline__ void cp_async4(float *dst, const float *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct NormIn {          // RMSNorm input of a NORM panel kernel
    const float *x;      // [n][cols] residual rows
    const float *w;      // [cols] norm multiplier
    float eps;
};

// RMSNorm + A8 of n rows into shared memory (pf_rmsnorm, forward_ops.c:191-200, then
// kern_quant_act). sx: [n][cols] fp32 and sw: [cols] already staged. Threads of the CTA.
__device__ __forceinline__ void norm_quant_smem(const float *sx, const float *sw, int n, int cols,
                                                float eps, int8_t *sq, float *sd, float *sfs, float *srr,
                                                int qstride = 0) {
    if (qstride == 0) qstride = cols;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    if (warp == 0) {
        // lanes 4v..4v+3: the four interleaved partial sums of row v (cols % 4 == 0)
        const int v = lane >> 2, l = lane & 3;
        float c = 0.0f;
        if (v < n) {
            const float *x = sx + (size_t)v * cols;
#pragma unroll 32
            for (int i = l; i < cols; i += 4) c = madd(c, x[i], x[i]);
        }
        const int base = lane & ~3;
        const float c0 = __shfl_sync(0xffffffffu, c, base), c1 = __shfl_sync(0xffffffffu, c, base + 1);
        const float c2 = __shfl_sync(0xffffffffu, c, base + 2), c3 = __shfl_sync(0xffffffffu, c, base + 3);
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
        if (v < n && l == 0) srr[v] = inv_sqrt_ref(__fadd_rn(__fdiv_rn(ss, (float)cols), eps));
    }
    __syncthreads();
    // A8: one thread per 32-column block (kern_quant_act: max, division, rounding and code sum
    // are order-independent, so the bits equal the warp-wide form). Thread t starts at 16-byte
    // chunk t % 8 of its block, so the 8 threads of a shared-memory phase read 8 distinct
    // bank groups although their blocks are 128 bytes apart.
    const int nb = cols >> 5;
    (void)lane;
    (void)warp;
    (void)nw;
    for (int u = tid; u < n * nb; u += blockDim.x) {
        const int v = u / nb, b = u % nb;
        const float r = srr[v];
        const float *xb = sx + (size_t)v * cols + b * 32, *wb = sw + b * 32;
        float xn[32];
        float a = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int ch = (k + tid) & 7;
            const float4 xv = *reinterpret_cast<const float4 *>(xb + 4 * ch);
            const float4 wv = *reinterpret_cast<const float4 *>(wb + 4 * ch);
            xn[4 * k + 0] = __fmul_rn(__fmul_rn(xv.x, r), wv.x);
            xn[4 * k + 1] = __fmul_rn(__fmul_rn(xv.y, r), wv.y);
            xn[4 * k + 2] = __fmul_rn(__fmul_rn(xv.z, r), wv.z);
            xn[4 * k + 3] = __fmul_rn(__fmul_rn(xv.w, r), wv.w);
            // fmaxf keeps the non-NaN operand: the max of the block's non-NaN |x|, NaN if all
            // are NaN, in any order (no seed value, as in the warp-wide form)
            const float m4 = fmaxf(fmaxf(fabsf(xn[4 * k]), fabsf(xn[4 * k + 1])),
                                   fmaxf(fabsf(xn[4 * k + 2]), fabsf(xn[4 * k + 3])));
            a = k == 0 ? m4 : fmaxf(a, m4);
        }
        const float id = a > 0.0f ? __fdiv_rn(127.0f, a) : 0.0f;
        int sum = 0;
        int8_t *qb = sq + (size_t)v * qstride + b * 32;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int ch = (k + tid) & 7;
            uint32_t packed = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int q = __float2int_rn(__fmul_rn(xn[4 * k + i], id));
                sum += q;
                packed |= (uint32_t)(uint8_t)(int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q)) << (8 * i);
            }
            *reinterpret_cast<uint32_t *>(qb + 4 * ch) = packed;
        }
        const float d = __fdiv_rn(a, 127.0f);
        sd[(size_t)v * nb + b] = d;
        sfs[(size_t)v * nb + b] = __fmul_rn(d, (float)sum);
    }
}

// One superblock of one row (this lane) for every vector: decode the 6-bit scales, integer
// block dots against the A8 activations (staged in shared memory), and the ordered fused chain
// into acc[v]. sq: [NMAX][cols] int8, sd / sfs: [NMAX][nb] block scales d and sums fsum.
template <int NMAX>
__device__ __forceinline__ void sb_accumulate(const uint4 sc, const uint4 (&cd)[8], const int8_t *sq,
                                              const float *sd, const float *sfs, int cols, int sb, int n,
                                              float (&acc)[NMAX]) {
    const int nb = cols >> 5;
    const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
    const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
    const float D = half_bits_to_float((uint32_t)(A >> 48));
    const float M = half_bits_to_float((uint32_t)(B >> 48));
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float ds = __fmul_rn(D, (float)(uint32_t)((A >> (6 * k)) & 63u));
        const float os = __fmul_rn(M, (float)(uint32_t)((B >> (6 * k)) & 63u));
        const int b = sb * 8 + k;
        const int lo0 = (int)(cd[k].x & 0x0f0f0f0fu), lo1 = (int)(cd[k].y & 0x0f0f0f0fu);
        const int lo2 = (int)(cd[k].z & 0x0f0f0f0fu), lo3 = (int)(cd[k].w & 0x0f0f0f0fu);
        const int hi0 = (int)((cd[k].x >> 4) & 0x0f0f0f0fu), hi1 = (int)((cd[k].y >> 4) & 0x0f0f0f0fu);
        const int hi2 = (int)((cd[k].z >> 4) & 0x0f0f0f0fu), hi3 = (int)((cd[k].w >> 4) & 0x0f0f0f0fu);
#pragma unroll
        for (int v = 0; v < NMAX; v++) {
            if (v < n) {
                const int4 *xq = reinterpret_cast<const int4 *>(sq + (size_t)v * cols + b * 32);
                const int4 x0 = xq[0], x1 = xq[1];
                int sacc = __dp4a(lo0, x0.x, 0);
                sacc = __dp4a(lo1, x0.y, sacc);
                sacc = __dp4a(lo2, x0.z, sacc);
                sacc = __dp4a(lo3, x0.w, sacc);
                sacc = __dp4a(hi0, x1.x, sacc);
                sacc = __dp4a(hi1, x1.y, sacc);
                sacc = __dp4a(hi2, x1.z, sacc);
                sacc = __dp4a(hi3, x1.w, sacc);
                acc[v] = __fmaf_rn((float)sacc, __fmul_rn(ds, sd[(size_t)v * nb + b]), acc[v]);
                acc[v] = __fmaf_rn(-os, sfs[(size_t)v * nb + b], acc[v]);
            }
        }
    }
}

// Activations of a panel / head kernel into shared memory by TMA bulk copies completing on
// `abar` (thread 0 issues them; every thread then waits): NORM the residual rows x [n][cols]
// fp32 and the norm weight [cols], else the A8 rows q [n][cols] and their block scales d and
// sums fsum [n][cols / 32]. Returns false if the wait timed out.
template <bool NORM>
__device__ __forceinline__ bool stage_act(uint64_t *abar, int n, int cols, const Act &in, const NormIn &nin,
                                          float *sx, float *sw, int8_t *sq, float *sd, float *sfs,
                                          int qstride = 0) {
    const int nb = cols >> 5;
    if (qstride == 0) qstride = cols;
    if (threadIdx.x == 0) {
        mbar_init(abar, 1);
        fence_mbar_init();
        if (NORM) {
            mbar_arrive_expect(abar, (uint32_t)(n + 1) * cols * 4u);
            bulk_g2s(sx, nin.x, (uint32_t)n * cols * 4u, abar);
            bulk_g2s(sw, nin.w, (uint32_t)cols * 4u, abar);
        } else {
            const int nbi = in.cols >> 5;
            mbar_arrive_expect(abar, (uint32_t)n * (cols + 8u * nb));
            for (int v = 0; v < n; v++) {
                bulk_g2s(sq + (size_t)v * qstride, in.q + (size_t)v * in.cols, (uint32_t)cols, abar);
                bulk_g2s(sd + (size_t)v * nb, in.d + (size_t)v * nbi, (uint32_t)nb * 4u, abar);
                bulk_g2s(sfs + (size_t)v * nb, in.fs + (size_t)v * nbi, (uint32_t)nb * 4u, abar);
            }
        }
    }
    __syncthreads();
    if (mbar_wait(abar, 0)) return true;
    mbar_wait(abar, 0);   // timed out: a second bounded wait lets the copies in flight land
    return false;
}

// An int loaded where it is written (volatile asm keeps its place among the other volatile asm),
// waited for only where it is used.
__device__ __forceinline__ int ld_early_s32(const int *p) {
    int v;
    asm volatile("ld.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_early_f32(const float *p) {
    float v;
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// After a timed-out wait on unit u of a warp's kRing-deep ring: units u .. u + kRing - 1 may
// still be in flight into this CTA's shared memory, so wait for each once more (bounded) before
// the warp returns.
__device__ __forceinline__ void drain_ring(uint64_t *bars, int u, int total) {
    for (int j = u; j < u + kRing && j < total; j++) mbar_wait(bars + j % kRing, (uint32_t)(j / kRing) & 1u);
}

size_t tall_smem(int cols, int nmax, bool norm) {
    size_t b = kTallSmem + (size_t)nmax * cols + (size_t)(cols / 32) * nmax * 8 + 16;
    b = (b + 15) & ~(size_t)15;
    if (norm) b += (size_t)nmax * cols * 4 + (size_t)cols * 4;
    return b;
}

// The tied LM head (248320 rows): persistent CTAs, a warp owns whole panels (lane = row) and
// walks their superblocks in column order through its TMA ring, so each (row, vector) chain
// stays in registers; logits (optional) and per-panel (max, first index) keys.
template <int NMAX, bool NORM>
__global__ void __launch_bounds__(kTallWarps * 32) k_mv_head(Mat W0, Act in, NormIn nin, Step *st,
                                                             float *y, int ldy,
                                                             unsigned long long *partial, int *nan0,
                                                             int row_base) {
    extern __shared__ __align__(128) uint8_t tsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *ring = tsm + (size_t)warp * kRing * kUnitBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(tsm + (size_t)kTallWarps * kRing * kUnitBytes) + warp * kRing;
    const int cols = W0.cols, nb = cols >> 5, nsb = W0.nsb;
    int8_t *sq = reinterpret_cast<int8_t *>(tsm + kTallSmem);
    float *sd = reinterpret_cast<float *>(tsm + kTallSmem + (size_t)NMAX * cols);   // [NMAX][nb]
    float *sfs = sd + (size_t)NMAX * nb;                                               // [NMAX][nb]
    uint64_t *abar = reinterpret_cast<uint64_t *>(sfs + (size_t)NMAX * nb);         // in the 16 B slack
    const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * kTallWarps;
    const int npw = W0.npanels > gw ? (W0.npanels - 1 - gw) / tw + 1 : 0;
    const int total = npw * nsb;
    auto src = [&](int u) -> const uint8_t * {
        const int panel = gw + (u / nsb) * tw;
        return W0.w + ((size_t)panel * nsb + (u % nsb)) * kUnitBytes;
    };
    if (lane == 0) {
        for (int i = 0; i < kRing; i++) mbar_init(bars + i, 1);
        fence_mbar_init();
        for (int u = 0; u < kRing && u < total; u++) tma_load_1d(ring + (size_t)u * kUnitBytes, src(u), kUnitBytes, bars + u);
    }
    pdl_wait();   // the ring above holds weights only
    pdl_trigger();
    const int n = st->n;
    if (n <= 0) {   // nothing to do: let the weight copies land before this CTA's shared memory goes
        __syncwarp();
        for (int u = 0; u < kRing && u < total; u++) mbar_wait(bars + u, 0);
        return;
    }
    // stage the activations while the first weight units are in flight: the A8 input, or
    // (NORM) the final RMSNorm of the residual rows computed here
    __shared__ float srr[NMAX];
    const size_t off = ((kTallSmem + (size_t)NMAX * cols + (size_t)nb * NMAX * 8 + 16) + 15) & ~(size_t)15;
    float *sx = reinterpret_cast<float *>(tsm + off), *sw = sx + (size_t)NMAX * cols;   // NORM only
    if (!stage_act<NORM>(abar, n, cols, in, nin, sx, sw, sq, sd, sfs) && threadIdx.x == 0)
        st->status = -90;   // device wait timed out: reported, no hang
    if (NORM) norm_quant_smem(sx, sw, n, cols, nin.eps, sq, sd, sfs, srr);
    __syncthreads();
    float acc[NMAX];
#pragma unroll
    for (int v = 0; v < NMAX; v++) acc[v] = 0.0f;
    for (int u = 0; u < total; u++) {
        const int slot = u % kRing;
        if (!mbar_wait(bars + slot, (uint32_t)(u / kRing) & 1u)) {
            if (lane == 0) st->status = -90;   // device wait timed out: reported, no hang
            drain_ring(bars, u, total);
            return;
        }
        const uint8_t *sp = ring + (size_t)slot * kUnitBytes + lane * 16;
        const uint4 sc = lds128(sp);
        uint4 cd[8];
#pragma unroll
        for (int k = 0; k < 8; k++) cd[k] = lds128(sp + 512 * (k + 1));
        __syncwarp();
        if (lane == 0 && u + kRing < total) {
            fence_proxy_async();
            tma_load_1d(ring + (size_t)slot * kUnitBytes, src(u + kRing), kUnitBytes, bars + slot);
        }
        const int sb = u % nsb;
        if (sb == 0) {
#pragma unroll
            for (int v = 0; v < NMAX; v++) acc[v] = 0.0f;
        }
        sb_accumulate<NMAX>(sc, cd, sq, sd, sfs, cols, sb, n, acc);
        if (sb != nsb - 1) continue;
        const int panel = gw + (u / nsb) * tw, row = panel * kPanelRows + lane;
#pragma unroll
        for (int v = 0; v < NMAX; v++) {
            if (v >= n) break;
            if (y && row < W0.rows) y[(size_t)v * ldy + row] = acc[v];
            const unsigned long long key = row < W0.rows ? argmax_key(acc[v], row_base + row) : 0ull;
            const unsigned long long best = warp_max_u64(key);
            if (lane == 0) partial[(size_t)v * W0.npanels + panel] = best;
            if (panel == 0 && lane == 0 && row_base == 0) nan0[v] = acc[v] != acc[v];
        }
    }
}

// The LM head for n <= 4 rows with the exact int8 block dots on the tensor cores.
// Same persistent schedule as k_mv_head (a warp owns whole panels and walks their units through a
// TMA ring) and the same float arithmetic, but each 32-row x 32-column block of a unit is one
// ldmatrix (the 16-byte row entries of rows 0..31) and two mma.sync.m16n8k32.s8 (rows 0-15 and
// 16-31) against the A8 activations, instead of 32 dp4a and 8 shared loads per row. MMA
// fragments: A row groupID (+8), columns 4 t..4 t+3 (+16) of the block = the low (high) nibbles
// of bytes 4 t..4 t+3 of the row entry, exactly one ldmatrix word; B column n = vector n & 3
// (columns 4..7 repeat vectors 0..3 so every lane receives useful sums); C: thread (g, t)
// takes rows g (t < 2) or g + 8 (t >= 2) of each half for vectors 2 (t & 1), 2 (t & 1) + 1.
// Integer sums are exact, so each (row, vector) chain
//   acc = fma((float)isum, (D s6) d, acc); acc = fma(-(M m6), fsum, acc)   (blocks in order)
// is bit-identical to kern_q4k and to k_mv_head. Then per-panel (max, first index) keys.
constexpr int kHeadQPad = 16;   // bytes of padding per activation row: conflict-free B loads

size_t head_mma_smem(int cols, bool norm) {
    const size_t nb = cols / 32;
    size_t b = kTallSmem + 16 + 4 * ((size_t)cols + kHeadQPad) + nb * 2 * 16 + 2 * 4 * nb * 4;
    b = (b + 15) & ~(size_t)15;
    if (norm) b += 4 * (size_t)cols * 4 + (size_t)cols * 4;
    return b;
}

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}

// fctr != nullptr (one context, unsharded head): the argmax is finished here as well. Each CTA
// folds its warps' running best keys per vector into fbest[v][cta]; the CTA whose increment of
// *fctr completes the grid reduces fbest and writes Step::argmax with pf_argmax's NaN rule (the
// keys order like pf_argmax: value, then lowest index), then resets the counter for the next
// launch.
template <bool NORM>
__global__ void __launch_bounds__(kTallWarps * 32) k_mv_head_mma(Mat W0, Act in, NormIn nin, Step *st,
                                                                 float *y, int ldy,
                                                                 unsigned long long *partial, int *nan0,
                                                                 int row_base, unsigned long long *fbest,
                                                                 int *fctr) {
    extern __shared__ __align__(128) uint8_t hsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3, tv = t & 1;   // MMA group / thread in group; vector pair
    uint8_t *ring = hsm + (size_t)warp * kRing * kUnitBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(hsm + (size_t)kTallWarps * kRing * kUnitBytes) + warp * kRing;
    const int cols = W0.cols, nb = cols >> 5, nsb = W0.nsb, qs = cols + kHeadQPad;
    uint64_t *abar = reinterpret_cast<uint64_t *>(hsm + kTallSmem);
    int8_t *sq = reinterpret_cast<int8_t *>(hsm + kTallSmem + 16);                  // [4][qs]
    float4 *sdfq = reinterpret_cast<float4 *>(sq + 4 * (size_t)qs);                 // [nb][2]
    float *sd = reinterpret_cast<float *>(sdfq + (size_t)nb * 2), *sfs = sd + 4 * (size_t)nb;
    const size_t off = (kTallSmem + 16 + 4 * (size_t)qs + (size_t)nb * 32 + 2 * 4 * (size_t)nb * 4 + 15) & ~(size_t)15;
    float *sx = reinterpret_cast<float *>(hsm + off), *sw = sx + 4 * (size_t)cols;   // NORM only
    const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * kTallWarps;
    const int npw = W0.npanels > gw ? (W0.npanels - 1 - gw) / tw + 1 : 0;
    const int total = npw * nsb;
    auto src = [&](int u) -> const uint8_t * {
        const int panel = gw + (u / nsb) * tw;
        return W0.w + ((size_t)panel * nsb + (u % nsb)) * kUnitBytes;
    };
    if (lane == 0) {
        for (int i = 0; i < kRing; i++) mbar_init(bars + i, 1);
        fence_mbar_init();
        for (int u = 0; u < kRing && u < total; u++) tma_load_1d(ring + (size_t)u * kUnitBytes, src(u), kUnitBytes, bars + u);
    }
    pdl_wait();   // the ring above holds weights only
    pdl_trigger();
    const int n = st->n;
    if (n <= 0) {   // nothing to do: let the weight copies land before this CTA's shared memory goes
        __syncwarp();
        for (int u = 0; u < kRing && u < total; u++) mbar_wait(bars + u, 0);
        return;
    }
    __shared__ float srr[4];
    if (!stage_act<NORM>(abar, n, cols, in, nin, sx, sw, sq, sd, sfs, qs) && threadIdx.x == 0)
        st->status = -90;   // device wait timed out: reported, no hang
    if (NORM) norm_quant_smem(sx, sw, n, cols, nin.eps, sq, sd, sfs, srr, qs);
    __syncthreads();
    // (d, fsum) of vectors 2 p and 2 p + 1 for block b at sdfq[2 b + p]
    for (int i = threadIdx.x; i < 2 * nb; i += blockDim.x) {
        const int b = i >> 1, p = i & 1;
        sdfq[i] = make_float4(sd[(2 * p) * nb + b], sfs[(2 * p) * nb + b], sd[(2 * p + 1) * nb + b],
                              sfs[(2 * p + 1) * nb + b]);
    }
    __syncthreads();
    const int8_t *bq = sq + (size_t)(g & 3) * qs + 4 * t;   // B fragment base of this lane
    const int r0 = (t < 2 ? 0 : 8) + g;                     // this lane's row in each 16-row half
    float acc[2][2];                                         // [half][vector of the pair]
    unsigned long long run[2] = {0ull, 0ull};               // best key so far of vector 2 tv + j
    for (int u = 0; u < total; u++) {
        const int slot = u % kRing;
        if (!mbar_wait(bars + slot, (uint32_t)(u / kRing) & 1u)) {
            if (lane == 0) st->status = -90;   // device wait timed out: reported, no hang
            drain_ring(bars, u, total);
            break;                             // (the fused argmax below still meets every CTA)
        }
        const uint8_t *sp = ring + (size_t)slot * kUnitBytes;
        const int sb = u % nsb;
        if (sb == 0) {
            acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.0f;
        }
        // scale entries of this lane's two rows
        const uint4 sc0 = lds128(sp + 16 * r0), sc1 = lds128(sp + 16 * (r0 + 16));
        const unsigned long long A0 = (unsigned long long)sc0.x | ((unsigned long long)sc0.y << 32);
        const unsigned long long B0 = (unsigned long long)sc0.z | ((unsigned long long)sc0.w << 32);
        const unsigned long long A1 = (unsigned long long)sc1.x | ((unsigned long long)sc1.y << 32);
        const unsigned long long B1 = (unsigned long long)sc1.z | ((unsigned long long)sc1.w << 32);
        const float D0 = half_bits_to_float((uint32_t)(A0 >> 48)), M0 = half_bits_to_float((uint32_t)(B0 >> 48));
        const float D1 = half_bits_to_float((uint32_t)(A1 >> 48)), M1 = half_bits_to_float((uint32_t)(B1 >> 48));
        uint32_t am[8][4];
#pragma unroll
        for (int k = 0; k < 8; k++) ldsm_x4(am[k], sp + 512 * (k + 1) + 16 * lane);
        __syncwarp();
        if (lane == 0 && u + kRing < total) {
            fence_proxy_async();
            tma_load_1d(ring + (size_t)slot * kUnitBytes, src(u + kRing), kUnitBytes, bars + slot);
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int b = sb * 8 + k;
            const uint32_t b0 = *reinterpret_cast<const uint32_t *>(bq + b * 32);
            const uint32_t b1 = *reinterpret_cast<const uint32_t *>(bq + b * 32 + 16);
            int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
            mma_s8_16832(c0, am[k][0] & 0x0f0f0f0fu, am[k][1] & 0x0f0f0f0fu, (am[k][0] >> 4) & 0x0f0f0f0fu,
                         (am[k][1] >> 4) & 0x0f0f0f0fu, b0, b1);
            mma_s8_16832(c1, am[k][2] & 0x0f0f0f0fu, am[k][3] & 0x0f0f0f0fu, (am[k][2] >> 4) & 0x0f0f0f0fu,
                         (am[k][3] >> 4) & 0x0f0f0f0fu, b0, b1);
            const float4 df = sdfq[2 * b + tv];
            const int i00 = t < 2 ? c0[0] : c0[2], i01 = t < 2 ? c0[1] : c0[3];
            const int i10 = t < 2 ? c1[0] : c1[2], i11 = t < 2 ? c1[1] : c1[3];
            const float ds0 = __fmul_rn(D0, (float)(uint32_t)((A0 >> (6 * k)) & 63u));
            const float os0 = __fmul_rn(M0, (float)(uint32_t)((B0 >> (6 * k)) & 63u));
            const float ds1 = __fmul_rn(D1, (float)(uint32_t)((A1 >> (6 * k)) & 63u));
            const float os1 = __fmul_rn(M1, (float)(uint32_t)((B1 >> (6 * k)) & 63u));
            acc[0][0] = __fmaf_rn((float)i00, __fmul_rn(ds0, df.x), acc[0][0]);
            acc[0][0] = __fmaf_rn(-os0, df.y, acc[0][0]);
            acc[0][1] = __fmaf_rn((float)i01, __fmul_rn(ds0, df.z), acc[0][1]);
            acc[0][1] = __fmaf_rn(-os0, df.w, acc[0][1]);
            acc[1][0] = __fmaf_rn((float)i10, __fmul_rn(ds1, df.x), acc[1][0]);
            acc[1][0] = __fmaf_rn(-os1, df.y, acc[1][0]);
            acc[1][1] = __fmaf_rn((float)i11, __fmul_rn(ds1, df.z), acc[1][1]);
            acc[1][1] = __fmaf_rn(-os1, df.w, acc[1][1]);
        }
        if (sb != nsb - 1) continue;
        // panel done: logits and the per-panel keys (rows r0 and r0 + 16, vectors 2 tv, 2 tv + 1)
        const int panel = gw + (u / nsb) * tw, rowa = panel * kPanelRows + r0, rowb = rowa + 16;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int v = 2 * tv + j;
            const bool live = v < n;
            if (live && y) {
                if (rowa < W0.rows) y[(size_t)v * ldy + rowa] = acc[0][j];
                if (rowb < W0.rows) y[(size_t)v * ldy + rowb] = acc[1][j];
            }
            const unsigned long long ka = rowa < W0.rows ? argmax_key(acc[0][j], row_base + rowa) : 0ull;
            const unsigned long long kb = rowb < W0.rows ? argmax_key(acc[1][j], row_base + rowb) : 0ull;
            unsigned long long best = ka > kb ? ka : kb;
            // lanes holding the same vector pair: t and t ^ 2 over every g
#pragma unroll
            for (int o = 2; o <= 16; o <<= 1) {
                const unsigned long long w = __shfl_xor_sync(0xffffffffu, best, o);
                best = w > best ? w : best;
            }
            if (live && lane == tv) partial[(size_t)v * W0.npanels + panel] = best;
            if (live && panel == 0 && lane == tv && row_base == 0) nan0[v] = acc[0][j] != acc[0][j];
            run[j] = best > run[j] ? best : run[j];
        }
    }
    if (fctr == nullptr) return;
    __shared__ unsigned long long s_best[kTallWarps][4];
    __shared__ int s_last;
    if (lane < 2) {   // lane tv holds vectors 2 tv and 2 tv + 1
        s_best[warp][2 * lane] = run[0];
        s_best[warp][2 * lane + 1] = run[1];
    }
    __syncthreads();
    if (threadIdx.x < 4) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kTallWarps; w++) b = s_best[w][threadIdx.x] > b ? s_best[w][threadIdx.x] : b;
        fbest[(size_t)threadIdx.x * gridDim.x + blockIdx.x] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(fctr, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (warp < n) {   // warp v finishes vector v
        unsigned long long b = 0ull;
        for (int i = lane; i < (int)gridDim.x; i += 32) {
            const unsigned long long k = __ldcg(fbest + (size_t)warp * gridDim.x + i);
            b = k > b ? k : b;
        }
        b = warp_max_u64(b);
        if (lane == 0) st->argmax[warp] = __ldcg(nan0 + warp) ? 0 : (int)(0xffffffffu - (uint32_t)(b & 0xffffffffu));
    }
    if (threadIdx.x == 0) *fctr = 0;
}

// Every matrix except the LM head: one CTA per 32-row panel, laid out for latency (a verify
// pass reads each 1-5 MB matrix once; the kernel's time is its chain of dependent steps, not
// the weight stream):
//   before pdl_wait  every superblock unit of the panel is requested with one TMA bulk copy
//                    into a slot of its own (weights are constants), and NORM stages the norm
//                    multiplier;
//   after pdl_wait   the pass's input rows are loaded with 16-byte loads by every thread beside
//                    the Step block (rows 0..NMAX-1 whatever the pass's row count: the buffers
//                    hold kMaxRows rows, rows past n are never used): the A8 input of the
//                    previous kernel, or (NORM) the residual rows, normalised and quantised here
//                    (pf_rmsnorm + kern_quant_act; every CTA computes the same bits);
//   units            each unit is split over 1, 2 or 4 warps by blocks; a warp decodes the
//                    scales of its blocks and forms the exact int32 block dots of every vector
//                    with no branch on the row count (the dp4a terms of a block are summed as two
//                    4-deep chains: integer addition is exact in any order);
//   chain            one warp per (matrix, vector) with lane = row runs the ordered fused chain
//                    acc = fmaf((float)isum, (D s6) d, acc); acc = fmaf(-(M m6), fsum, acc)
//                    over the blocks in column order, its operands loaded eight blocks ahead;
//   epilogue         EPI 0: y[v][row] = acc (projections feeding DeltaNet / attention)
//                    EPI 1: y[v][row] += acc (out_proj / o_proj / down_proj into the residual)
//                    EPI 3: SwiGLU over (W0 = gate, W1 = up), the up accumulators handed to
//                    the gate warps through shared memory, then A8 of the product for down_proj.
// nmax <= 4. Block: 16 warps (8 for one-row passes of up to 8 units).
constexpr int kPanelWarps = 16;
constexpr int kPanelPad = 4;   // fp32 row padding of the staged residual rows (bank spread)

struct PanelSmem {             // byte offsets into the dynamic shared memory
    size_t bars, isum, ds, os, sd, sfs, sq, sx, sw, sg, total;
};
__host__ __device__ inline PanelSmem panel_layout(int nunit, int cols, int nmat, int nmax, bool norm) {
    PanelSmem L;
    const size_t nb = cols / 32;
    size_t o = (size_t)nunit * kUnitBytes;
    L.bars = o;
    o += (((size_t)nunit + 1) * 8 + 15) & ~(size_t)15;
    L.isum = o;
    o += (size_t)nmat * nb * nmax * 32 * 4;
    L.ds = o;
    o += (size_t)nmat * nb * 32 * 4;
    L.os = o;
    o += (size_t)nmat * nb * 32 * 4;
    L.sd = o;
    o += (size_t)nmax * nb * 4;
    L.sfs = o;
    o += (size_t)nmax * nb * 4;
    L.sq = o;
    o += (size_t)nmax * cols;
    o = (o + 15) & ~(size_t)15;
    L.sx = o;
    if (norm) o += (size_t)nmax * (cols + kPanelPad) * 4;
    L.sw = o;
    if (norm) o += (size_t)cols * 4;
    L.sg = o;
    o += (size_t)nmax * 32 * 4;
    L.total = o;
    return L;
}

// RMSNorm + A8 of the staged rows (pf_rmsnorm, forward_ops.c:191-200, then kern_quant_act):
// sx [NMAX][cols + kPanelPad] fp32, sw [cols]; writes sq [NMAX][cols], sd / sfs [NMAX][cols/32].
// The sum of squares keeps the reference's four interleaved lane sums (lane l adds x[l], x[l+4],
// ... in order): lanes 4v..4v+3 of warp 0 (the padded row stride puts the 16 lanes on distinct
// banks). The A8 takes four threads per
// 32-column block, eight columns each: max, division, rounding and code sum are
// order-independent, so the bits equal the warp-wide quantiser's.
template <int NMAX>
__device__ __forceinline__ void panel_norm_quant(const float *sx, const float *sw, int cols, float eps,
                                                 int8_t *sq, float *sd, float *sfs, float *srr) {
    const int tid = threadIdx.x, xs = cols + kPanelPad;
    if (tid < 4 * NMAX) {
        const int v = tid >> 2, l = tid & 3;
        const float *x = sx + (size_t)v * xs + l;
        float c = 0.0f;
#pragma unroll 32
        for (int i = 0; i < cols; i += 4) c = madd(c, x[i], x[i]);
        const int base = tid & ~3;
        const unsigned m = (4 * NMAX >= 32) ? 0xffffffffu : ((1u << (4 * NMAX)) - 1u);
        const float c0 = __shfl_sync(m, c, base), c1 = __shfl_sync(m, c, base + 1);
        const float c2 = __shfl_sync(m, c, base + 2), c3 = __shfl_sync(m, c, base + 3);
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
        if (l == 0) srr[v] = inv_sqrt_ref(__fadd_rn(__fdiv_rn(ss, (float)cols), eps));
    }
    __syncthreads();
    // A8: one thread per 32-column block, starting at 16-byte chunk t % 8 of its block so the 8
    // threads of a shared-memory phase read 8 distinct bank groups
    const int nb = cols >> 5;
    for (int u = tid; u < NMAX * nb; u += blockDim.x) {
        const int v = u / nb, b = u - v * nb;
        const float r = srr[v];
        const float *xb = sx + (size_t)v * xs + b * 32, *wb = sw + b * 32;
        float xn[32];
        float a = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int ch = (k + tid) & 7;
            const float4 xv = *reinterpret_cast<const float4 *>(xb + 4 * ch);
            const float4 wv = *reinterpret_cast<const float4 *>(wb + 4 * ch);
            xn[4 * k + 0] = __fmul_rn(__fmul_rn(xv.x, r), wv.x);
            xn[4 * k + 1] = __fmul_rn(__fmul_rn(xv.y, r), wv.y);
            xn[4 * k + 2] = __fmul_rn(__fmul_rn(xv.z, r), wv.z);
            xn[4 * k + 3] = __fmul_rn(__fmul_rn(xv.w, r), wv.w);
            // fmaxf keeps the non-NaN operand: the max of the block's non-NaN |x|, NaN if all
            // are NaN, in any order (as the warp-wide form)
            const float m4 = fmaxf(fmaxf(fabsf(xn[4 * k]), fabsf(xn[4 * k + 1])),
                                   fmaxf(fabsf(xn[4 * k + 2]), fabsf(xn[4 * k + 3])));
            a = k == 0 ? m4 : fmaxf(a, m4);
        }
        const float id = a > 0.0f ? __fdiv_rn(127.0f, a) : 0.0f;
        int sum = 0;
        int8_t *qb = sq + (size_t)v * cols + b * 32;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int ch = (k + tid) & 7;
            uint32_t packed = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int q = __float2int_rn(__fmul_rn(xn[4 * k + i], id));
                sum += q;
                packed |= (uint32_t)(uint8_t)(int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q)) << (8 * i);
            }
            *reinterpret_cast<uint32_t *>(qb + 4 * ch) = packed;
        }
        const float d = __fdiv_rn(a, 127.0f);
        sd[(size_t)v * nb + b] = d;
        sfs[(size_t)v * nb + b] = __fmul_rn(d, (float)sum);
    }
}

// ---- staging of a pass's input rows into shared memory, after pdl_wait
// A segment is `rows` rows of `per` 16-byte chunks. Each row gets blockDim / rows threads (rows
// divides the block), and thread t of a row takes chunks t, t + TPR, ...: no division per chunk.
// Every load of a thread (up to 4 chunks of the first segment and one of each of the others) is
// issued, volatile and so in program order, before its first store, so the rows arrive in one
// round trip to L2 (the compiler cannot tell the shared destination from the global source).
struct StageSeg {
    uint8_t *dst;
    const uint8_t *src;
    int dstride, sstride;   // bytes between rows
    int per, rows;          // 16-byte chunks per row, rows
};
__device__ __forceinline__ uint4 ld_early_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
// a: the main segment; b, c: small segments of the same row count with per <= blockDim / rows
// (b.rows == 0: none)
__device__ __forceinline__ void stage_rows3(const StageSeg &a, const StageSeg &b, const StageSeg &c) {
    const int tpr = (int)blockDim.x / a.rows, v = (int)threadIdx.x / tpr, c0 = (int)threadIdx.x - v * tpr;
    uint4 ra[4], rb, rc;
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (c0 + j * tpr < a.per) ra[j] = ld_early_v4(a.src + (size_t)v * a.sstride + 16 * (c0 + j * tpr));
    const bool hb = b.rows > 0 && c0 < b.per, hc = c.rows > 0 && c0 < c.per;
    if (hb) rb = ld_early_v4(b.src + (size_t)v * b.sstride + 16 * c0);
    if (hc) rc = ld_early_v4(c.src + (size_t)v * c.sstride + 16 * c0);
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (c0 + j * tpr < a.per)
            *reinterpret_cast<uint4 *>(a.dst + (size_t)v * a.dstride + 16 * (c0 + j * tpr)) = ra[j];
    if (hb) *reinterpret_cast<uint4 *>(b.dst + (size_t)v * b.dstride + 16 * c0) = rb;
    if (hc) *reinterpret_cast<uint4 *>(c.dst + (size_t)v * c.dstride + 16 * c0) = rc;
    for (int k = c0 + 4 * tpr; k < a.per; k += tpr)   // rows longer than 4 chunks per thread
        *reinterpret_cast<uint4 *>(a.dst + (size_t)v * a.dstride + 16 * k) =
            ld_early_v4(a.src + (size_t)v * a.sstride + 16 * k);
}

// This CTA's share of the L2 prefetch ranges: the concatenated ranges split evenly (16-byte
// granules) over the grid, one bulk prefetch per range piece.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch &pf, const Step *st) {
    if (pf.n == 0 || threadIdx.x != 0) return;
    unsigned len[kMaxPrefetch];
    unsigned long long total = 0;
    int rows = -1;
    for (int i = 0; i < pf.n; i++) {
        len[i] = pf.bytes[i];
        if (pf.row_bytes[i]) {   // a KV cache: the rows up to the pass's last position
            if (rows < 0) rows = st->pos0 + st->n;
            const unsigned long long want = (unsigned long long)(rows > 0 ? rows : 0) * pf.row_bytes[i];
            len[i] = (unsigned)((want < len[i] ? want : len[i]) & ~15ull);
        }
        total += len[i];
    }
    const unsigned long long g = total >> 4, G = gridDim.x, c = blockIdx.x;
    unsigned long long lo = (g * c / G) << 4, hi = (g * (c + 1) / G) << 4, base = 0;
    for (int i = 0; i < pf.n && lo < hi; i++) {
        const unsigned long long e = base + len[i];
        if (lo < e) {
            const unsigned long long a = lo, b = hi < e ? hi : e;
            const char *src = static_cast<const char *>(pf.p[i]) + (a - base);
            for (unsigned long long o = 0; o < b - a; o += 65536) {
                const unsigned sz = (unsigned)((b - a - o) < 65536 ? (b - a - o) : 65536);
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src + o), "r"(sz) : "memory");
            }
            lo = b;
        }
        base = e;
    }
}

// PPC: panels per CTA for EPI 0 (2 when the matrix has more panels than the GPU has SMs, so
// the CTAs fit beside the previous kernel's); EPI 1 / 3 take one.
template <int NMAX, int EPI, bool NORM, int PPC = 1>
__global__ void __launch_bounds__(kPanelWarps * 32) k_mv_panel(Mat W0, Mat W1, Act in, NormIn nin,
                                                               Step *st, float *y, int ldy, Act out,
                                                               L2Prefetch pf) {
    static_assert(PPC == 1 || (PPC == 2 && EPI == 0), "two panels per CTA for EPI 0 only");
    extern __shared__ __align__(128) uint8_t wsm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int nsb = W0.nsb, cols = W0.cols, nb = cols >> 5, panel = blockIdx.x * PPC;
    constexpr int nmat = EPI == 3 ? 2 : PPC;   // unit groups: gate / up, or this CTA's panels
    // the panel of unit group m, and whether it exists (a last CTA may have one panel of two)
    auto gpanel = [&](int m) { return PPC == 2 ? panel + m : panel; };
    auto gmat = [&](int m) -> const Mat & { return (EPI == 3 && m) ? W1 : W0; };
    const int nunit = nsb * nmat;
    const PanelSmem PL = panel_layout(nunit, cols, nmat, NMAX, NORM);
    uint8_t *units = wsm;
    uint64_t *bars = reinterpret_cast<uint64_t *>(wsm + PL.bars);
    int32_t *isum = reinterpret_cast<int32_t *>(wsm + PL.isum);   // [nmat][nb][NMAX][32]
    float *ds = reinterpret_cast<float *>(wsm + PL.ds);           // [nmat][nb][32]
    float *os = reinterpret_cast<float *>(wsm + PL.os);
    float *sd = reinterpret_cast<float *>(wsm + PL.sd);           // [NMAX][nb]
    float *sfs = reinterpret_cast<float *>(wsm + PL.sfs);
    int8_t *sq = reinterpret_cast<int8_t *>(wsm + PL.sq);          // [NMAX][cols]
    float *sx = reinterpret_cast<float *>(wsm + PL.sx);           // NORM: [NMAX][cols + pad]
    float *sw = reinterpret_cast<float *>(wsm + PL.sw);           // NORM: [cols]
    float *sg = reinterpret_cast<float *>(wsm + PL.sg);           // EPI 3: [NMAX][32]
    __shared__ float srr[NMAX];
    // thread u requests unit u (weights: safe before pdl_wait)
    if (tid < nunit && gpanel(tid / nsb) < W0.npanels) {
        const int m = tid / nsb, sb = tid % nsb;
        mbar_init(bars + tid, 1);
        fence_mbar_init();
        tma_load_1d(units + (size_t)tid * kUnitBytes, gmat(m).w + ((size_t)gpanel(m) * nsb + sb) * kUnitBytes,
                    kUnitBytes, bars + tid);
    }
    if (NORM) {   // the norm multiplier (constant: safe before pdl_wait)
        for (int i = tid; i < cols / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(sw)[i] = reinterpret_cast<const float4 *>(nin.w)[i];
    }
    l2_prefetch_share(pf, st);   // weights and KV rows of kernels further ahead
    pdl_wait();
    pdl_trigger();
    const int n = ld_early_s32(&st->n);
    if (NORM) {   // the residual rows beside the Step block
        if (NMAX == 1) {   // one row: all of it at once (measured faster for one-row passes)
            const StageSeg none{};
            stage_rows3({reinterpret_cast<uint8_t *>(sx), reinterpret_cast<const uint8_t *>(nin.x),
                         (cols + kPanelPad) * 4, cols * 4, cols / 4, NMAX}, none, none);
        } else {   // several rows, which 100+ CTAs read at once: one chunk after another per thread,
                   // which spreads the requests for the same lines (measured faster than a burst)
            const int per = cols / 4, total = NMAX * per;
            for (int i = tid; i < total; i += blockDim.x) {
                const int v = i / per, c4 = i - v * per;
                reinterpret_cast<float4 *>(sx + (size_t)v * (cols + kPanelPad))[c4] =
                    reinterpret_cast<const float4 *>(nin.x + (size_t)v * cols)[c4];
            }
        }
    } else {      // the A8 rows of the previous kernel beside the Step block
        const int nbi = in.cols >> 5;
        if (NMAX == 1) {
            stage_rows3({reinterpret_cast<uint8_t *>(sq), reinterpret_cast<const uint8_t *>(in.q), cols, in.cols, cols / 16, NMAX},
                        {reinterpret_cast<uint8_t *>(sd), reinterpret_cast<const uint8_t *>(in.d), nb * 4, nbi * 4, nb / 4, NMAX},
                        {reinterpret_cast<uint8_t *>(sfs), reinterpret_cast<const uint8_t *>(in.fs), nb * 4, nbi * 4, nb / 4, NMAX});
        } else {
            const int per = cols / 16;
            for (int i = tid; i < NMAX * per; i += blockDim.x) {
                const int v = i / per, c16 = i - v * per;
                reinterpret_cast<int4 *>(sq + (size_t)v * cols)[c16] =
                    reinterpret_cast<const int4 *>(in.q + (size_t)v * in.cols)[c16];
            }
            const int per4 = nb / 4;
            for (int i = tid; i < NMAX * per4; i += blockDim.x) {
                const int v = i / per4, b4 = i - v * per4;
                reinterpret_cast<float4 *>(sd + (size_t)v * nb)[b4] = reinterpret_cast<const float4 *>(in.d + (size_t)v * nbi)[b4];
                reinterpret_cast<float4 *>(sfs + (size_t)v * nb)[b4] = reinterpret_cast<const float4 *>(in.fs + (size_t)v * nbi)[b4];
            }
        }
    }
    __syncthreads();
    if (n <= 0) {   // nothing to do: the weight copies land before this CTA's shared memory goes
        if (tid < nunit && gpanel(tid / nsb) < W0.npanels) mbar_wait(bars + tid, 0);
        return;
    }
    if (NORM) {
        panel_norm_quant<NMAX>(sx, sw, cols, nin.eps, sq, sd, sfs, srr);
        __syncthreads();
    }
    // ---- units: task = (unit, part), part = a run of 8 / sp blocks
    const int sp = nunit * 4 <= nw ? 4 : (nunit * 2 <= nw ? 2 : 1), kb = 8 / sp;
    for (int task = warp; task < nunit * sp; task += nw) {
        const int u = task / sp, part = task - u * sp, m = u / nsb, sb = u - m * nsb;
        if (gpanel(m) >= W0.npanels) continue;
        if (!mbar_wait(bars + u, 0)) {
            if (lane == 0) st->status = -90;   // device wait timed out: reported, no hang
            mbar_wait(bars + u, 0);            // the unit in flight lands before the warp goes
            continue;
        }
        const uint8_t *sp_ = units + (size_t)u * kUnitBytes + lane * 16;
        const uint4 sc = lds128(sp_);
        const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
        const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
        const float D = half_bits_to_float((uint32_t)(A >> 48));
        const float M = half_bits_to_float((uint32_t)(B >> 48));
        for (int kk = 0; kk < kb; kk++) {
            const int k = part * kb + kk, b = sb * 8 + k;
            const uint4 cd = lds128(sp_ + 512 * (k + 1));
            ds[((size_t)m * nb + b) * 32 + lane] = __fmul_rn(D, (float)(uint32_t)((A >> (6 * k)) & 63u));
            os[((size_t)m * nb + b) * 32 + lane] = __fmul_rn(M, (float)(uint32_t)((B >> (6 * k)) & 63u));
            const int lo0 = (int)(cd.x & 0x0f0f0f0fu), lo1 = (int)(cd.y & 0x0f0f0f0fu);
            const int lo2 = (int)(cd.z & 0x0f0f0f0fu), lo3 = (int)(cd.w & 0x0f0f0f0fu);
            const int hi0 = (int)((cd.x >> 4) & 0x0f0f0f0fu), hi1 = (int)((cd.y >> 4) & 0x0f0f0f0fu);
            const int hi2 = (int)((cd.z >> 4) & 0x0f0f0f0fu), hi3 = (int)((cd.w >> 4) & 0x0f0f0f0fu);
            int32_t *is = isum + ((size_t)m * nb + b) * NMAX * 32 + lane;
#pragma unroll
            for (int v = 0; v < NMAX; v++) {   // every vector: rows past n give unused sums
                const int4 *xq = reinterpret_cast<const int4 *>(sq + (size_t)v * cols + b * 32);
                const int4 x0 = xq[0], x1 = xq[1];
                int sl = __dp4a(lo0, x0.x, 0);
                int sh = __dp4a(hi0, x1.x, 0);
                sl = __dp4a(lo1, x0.y, sl);
                sh = __dp4a(hi1, x1.y, sh);
                sl = __dp4a(lo2, x0.z, sl);
                sh = __dp4a(hi2, x1.z, sh);
                sl = __dp4a(lo3, x0.w, sl);
                sh = __dp4a(hi3, x1.w, sh);
                is[v * 32] = sl + sh;
            }
        }
    }
    __syncthreads();
    // ---- chains: warp (m, v), lane = row
    const int m = warp / NMAX, v = warp - m * NMAX;
    const int row = gpanel(m) * kPanelRows + lane;
    const bool chain = warp < nmat * NMAX && v < n && gpanel(m) < W0.npanels;
    float acc = 0.0f;
    if (chain) {
        const float y_old = (EPI == 1 && row < W0.rows) ? ld_early_f32(y + (size_t)v * ldy + row) : 0.0f;
        const int32_t *is = isum + ((size_t)m * nb * NMAX + v) * 32 + lane;
        const float *dsp = ds + (size_t)m * nb * 32 + lane, *osp = os + (size_t)m * nb * 32 + lane;
        const float *dv = sd + (size_t)v * nb, *fv = sfs + (size_t)v * nb;
        float PA[8], QA[8], OA[8], FA[8], PB[8], QB[8], OB[8], FB[8];
#define NB_CHAIN_LOAD(P, Q, O, F, b0)                                                         \
        _Pragma("unroll") for (int j = 0; j < 8; j++) {                                      \
            P[j] = (float)is[(size_t)((b0) + j) * NMAX * 32];                                \
            Q[j] = __fmul_rn(dsp[((b0) + j) * 32], dv[(b0) + j]);                              \
            O[j] = osp[((b0) + j) * 32];                                                      \
            F[j] = fv[(b0) + j];                                                              \
        }
#define NB_CHAIN_RUN(P, Q, O, F)                                                              \
        _Pragma("unroll") for (int j = 0; j < 8; j++) {                                      \
            acc = __fmaf_rn(P[j], Q[j], acc);                                                 \
            acc = __fmaf_rn(-O[j], F[j], acc);                                                \
        }
        NB_CHAIN_LOAD(PA, QA, OA, FA, 0)
        for (int b0 = 0; b0 < nb; b0 += 16) {   // nb is a multiple of 8
            if (b0 + 8 < nb) { NB_CHAIN_LOAD(PB, QB, OB, FB, b0 + 8) }
            NB_CHAIN_RUN(PA, QA, OA, FA)
            if (b0 + 16 < nb) { NB_CHAIN_LOAD(PA, QA, OA, FA, b0 + 16) }
            if (b0 + 8 < nb) { NB_CHAIN_RUN(PB, QB, OB, FB) }
        }
#undef NB_CHAIN_LOAD
#undef NB_CHAIN_RUN
        if (EPI == 0 && row < W0.rows) y[(size_t)v * ldy + row] = acc;
        if (EPI == 1 && row < W0.rows) y[(size_t)v * ldy + row] = __fadd_rn(y_old, acc);
        if (EPI == 3 && m == 1) sg[v * 32 + lane] = acc;   // up, for the gate warp of vector v
    }
    if (EPI == 3) {
        __syncthreads();
        if (chain && m == 0) {
            const float h = __fmul_rn(pf_silu(acc), sg[v * 32 + lane]);
            const int nbo = out.cols >> 5;
            quant_block_warp(h, lane, out.q + (size_t)v * out.cols + panel * 32,
                             out.d + (size_t)v * nbo + panel, out.fs + (size_t)v * nbo + panel);
        }
    }
}


// The same matvec for matrices with long chains (out_proj / o_proj / down_proj: 1024 rows, 64 to
// 112 blocks per row), one CTA per 8-row slice of a panel (four CTAs share a panel), laid out so
// that every phase but the ordered chain runs on all 16 warps:
//   before pdl_wait  this slice of every unit (the 8 rows' scale entries and code entries: nine
//                    128-byte bulk copies per unit);
//   after pdl_wait   the A8 rows of the previous kernel, 16-byte loads spread over the CTA;
//   operands         (block, lane) items over all warps, lane = (vector v = lane / 8, row r =
//                    lane % 8): the exact int32 block dot and the four operands of the block's
//                    two chain steps, {(float)isum, (D s6) d, -(M m6), fsum}, one float4 per item;
//   chain            warp 0 runs the 32 ordered chains of the slice, one 16-byte shared-memory
//                    load and two dependent fmaf per block (the result is independent of where
//                    the operands were formed: the same roundings in the same order).
// EPI 0 / 1 as k_mv_panel; NMAX = 4.
constexpr int kSliceRows = 8;
constexpr int kSliceBytes = 9 * 128;   // per unit: scale entries + 8 blocks of code entries
constexpr int kSliceWarps = 16;
constexpr int kSlicePad = 16;          // bytes between the staged A8 rows (bank spread)

struct SliceSmem {
    size_t bars, ops, sd, sfs, sq, total;
};
__host__ __device__ inline SliceSmem slice_layout(int nunit, int cols) {
    SliceSmem L;
    const size_t nb = cols / 32;
    size_t o = (size_t)nunit * kSliceBytes;
    L.bars = o;
    o += (((size_t)nunit) * 8 + 15) & ~(size_t)15;
    L.ops = o;
    o += nb * 32 * 16;
    L.sd = o;
    o += 4 * (nb + 4) * 4;
    L.sfs = o;
    o += 4 * (nb + 4) * 4;
    L.sq = o;
    o += 4 * ((size_t)cols + kSlicePad);
    L.total = (o + 15) & ~(size_t)15;
    return L;
}

template <int EPI>
__global__ void __launch_bounds__(kSliceWarps * 32) k_mv_slice(Mat W0, Act in, Step *st, float *y, int ldy) {
    extern __shared__ __align__(128) uint8_t ssm[];
    constexpr int NMAX = 4;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nsb = W0.nsb, cols = W0.cols, nb = cols >> 5, nunit = nsb, nbp = nb + 4, qs = cols + kSlicePad;
    const int panel = blockIdx.x >> 2, r0 = (blockIdx.x & 3) * kSliceRows;
    const SliceSmem SL = slice_layout(nunit, cols);
    uint8_t *units = ssm;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ssm + SL.bars);
    float4 *ops = reinterpret_cast<float4 *>(ssm + SL.ops);       // [nb][32 lanes]
    float *sd = reinterpret_cast<float *>(ssm + SL.sd);           // [NMAX][nb + 4]
    float *sfs = reinterpret_cast<float *>(ssm + SL.sfs);
    int8_t *sq = reinterpret_cast<int8_t *>(ssm + SL.sq);          // [NMAX][cols + pad]
    // thread u copies its slice of unit u (weights: safe before pdl_wait)
    if (tid < nunit) {
        const uint8_t *src = W0.w + ((size_t)panel * nsb + tid) * kUnitBytes + r0 * 16;
        uint8_t *dst = units + (size_t)tid * kSliceBytes;
        mbar_init(bars + tid, 1);
        fence_mbar_init();
        mbar_arrive_expect(bars + tid, kSliceBytes);
        for (int p = 0; p < 9; p++) bulk_g2s(dst + p * 128, src + p * 512, 128, bars + tid);
    }
    pdl_wait();
    pdl_trigger();
    const int n = ld_early_s32(&st->n);
    {   // the A8 rows of the previous kernel beside the Step block
        const int nbi = in.cols >> 5;
        // one chunk after another per thread: 128 CTAs read the same rows at once, and spreading
        // the requests measured faster than issuing them in one burst
        const int per = cols / 16, per4 = nb / 4;
        for (int i = tid; i < NMAX * per; i += blockDim.x) {
            const int v = i / per, c16 = i - v * per;
            reinterpret_cast<int4 *>(sq + (size_t)v * qs)[c16] = reinterpret_cast<const int4 *>(in.q + (size_t)v * in.cols)[c16];
        }
        for (int i = tid; i < 2 * NMAX * per4; i += blockDim.x) {
            const int which = i / (NMAX * per4), j = i - which * NMAX * per4, v = j / per4, b4 = j - v * per4;
            const float *src = (which ? in.fs : in.d) + (size_t)v * nbi;
            float *dst = (which ? sfs : sd) + (size_t)v * nbp;
            reinterpret_cast<float4 *>(dst)[b4] = reinterpret_cast<const float4 *>(src)[b4];
        }
    }
    if (tid < nunit && !mbar_wait(bars + tid, 0)) {   // every unit in shared memory
        st->status = -90;                                // device wait timed out: reported, no hang
        mbar_wait(bars + tid, 0);                        // the copies in flight land before the CTA goes
    }
    __syncthreads();
    if (n <= 0) return;
    // ---- operands: item (block b, lane)
    const int v = lane >> 3, r = lane & 7;
    for (int b = warp; b < nb; b += kSliceWarps) {
        const int u = b >> 3, k = b & 7;
        const uint8_t *up = units + (size_t)u * kSliceBytes;
        const uint4 sc = lds128(up + r * 16);
        const uint4 cd = lds128(up + 128 * (k + 1) + r * 16);
        const int4 *xq = reinterpret_cast<const int4 *>(sq + (size_t)v * qs + b * 32);
        const int4 x0 = xq[0], x1 = xq[1];
        int sl = __dp4a((int)(cd.x & 0x0f0f0f0fu), x0.x, 0);
        int sh = __dp4a((int)((cd.x >> 4) & 0x0f0f0f0fu), x1.x, 0);
        sl = __dp4a((int)(cd.y & 0x0f0f0f0fu), x0.y, sl);
        sh = __dp4a((int)((cd.y >> 4) & 0x0f0f0f0fu), x1.y, sh);
        sl = __dp4a((int)(cd.z & 0x0f0f0f0fu), x0.z, sl);
        sh = __dp4a((int)((cd.z >> 4) & 0x0f0f0f0fu), x1.z, sh);
        sl = __dp4a((int)(cd.w & 0x0f0f0f0fu), x0.w, sl);
        sh = __dp4a((int)((cd.w >> 4) & 0x0f0f0f0fu), x1.w, sh);
        const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
        const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
        const float D = half_bits_to_float((uint32_t)(A >> 48));
        const float M = half_bits_to_float((uint32_t)(B >> 48));
        const float dsc = __fmul_rn(D, (float)(uint32_t)((A >> (6 * k)) & 63u));
        const float osc = __fmul_rn(M, (float)(uint32_t)((B >> (6 * k)) & 63u));
        ops[b * 32 + lane] = make_float4((float)(sl + sh), __fmul_rn(dsc, sd[v * nbp + b]), -osc, sfs[v * nbp + b]);
    }
    __syncthreads();
    // ---- the ordered chains: warp 0, lane (v, r)
    if (warp != 0) return;
    const int row = panel * kPanelRows + r0 + r;
    const bool live = v < n && row < W0.rows;
    const float y_old = (EPI == 1 && live) ? ld_early_f32(y + (size_t)v * ldy + row) : 0.0f;
    const float4 *op = ops + lane;
    float acc = 0.0f;
#pragma unroll 8
    for (int b = 0; b < nb; b++) {
        const float4 f = op[b * 32];
        acc = __fmaf_rn(f.x, f.y, acc);
        acc = __fmaf_rn(f.z, f.w, acc);
    }
    if (live) y[(size_t)v * ldy + row] = EPI == 1 ? __fadd_rn(y_old, acc) : acc;
}

size_t slice_smem(int nunit, int cols) { return slice_layout(nunit, cols).total; }

size_t panel_smem(int nunit, int cols, int nmat, int nmax, bool norm) {
    return panel_layout(nunit, cols, nmat, nmax, norm).total;
}

// ------------------------------------------------------------------ argmax over the panels
// Vocab-sharded head: this GPU's best key per verify row and its row-0 NaN flag, for the
// all-reduce (max) across the shards; k_keys_argmax turns the merged keys into tokens exactly
// as k_argmax_final does.
// keys: [best key of row r][NaN flag of row r] with the flags kstride after the keys; blockIdx.y
// = the sequence of a multi-sequence pass (row r = its row0 + v)
__global__ void k_argmax_keys(const unsigned long long *partial, const int *nan0, int npanels,
                              const Step *st, unsigned long long *keys, int kstride) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.y;
    const int v = blockIdx.x;
    if (v >= st->n) return;
    const int row = st->row0 + v;
    __shared__ unsigned long long red[32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < npanels; i += blockDim.x) {
        const unsigned long long k = partial[(size_t)row * npanels + i];
        best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        unsigned long long b = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
        b = warp_max_u64(b);
        if (threadIdx.x == 0) {
            keys[row] = b;
            keys[kstride + row] = nan0[row] ? 1ull : 0ull;
        }
    }
}
__global__ void k_keys_argmax(const unsigned long long *keys, Step *st, int kstride) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.x;   // the sequence of a multi-sequence pass
    const int v = threadIdx.x;
    if (v >= st->n) return;
    const int row = st->row0 + v;
    st->argmax[v] = keys[kstride + row] ? 0 : (int)(0xffffffffu - (uint32_t)(keys[row] & 0xffffffffu));
}

__global__ void k_argmax_final(const unsigned long long *partial, const int *nan0, int npanels,
                               Step *st) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.y;   // the sequence (multi-sequence passes)
    const int v = blockIdx.x;
    if (v >= st->n) return;
    const int row = st->row0 + v;
    __shared__ unsigned long long red[32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < npanels; i += blockDim.x) {
        const unsigned long long k = partial[(size_t)row * npanels + i];
        best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        unsigned long long b = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
        b = warp_max_u64(b);
        if (threadIdx.x == 0)
            st->argmax[v] = nan0[row] ? 0 : (int)(0xffffffffu - (uint32_t)(b & 0xffffffffu));
    }
}

// ------------------------------------------------------------------ embedding rows
// kern_get_row_q, Q4K branch (engine/src/kern_act.c:76-85): dd = D * s6, mm = M * m6,
// x = dd * u - mm (two roundings), read from the panel layout.
__global__ void k_embed(Mat E, const Step *st, float *x, int H) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.y;   // the sequence (multi-sequence passes)
    const int v = blockIdx.x;
    if (v >= st->n) return;
    const int row = st->row0 + v;
    int tok = st->tokens[v];
    if (tok < 0 || tok >= E.rows) tok = 0;   // host and accept kernel validate ids
    const int panel = tok >> 5, r = tok & 31;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        const int sb = c >> 8, k = (c >> 5) & 7, j = c & 31;
        const uint8_t *u = E.w + ((size_t)panel * E.nsb + sb) * kUnitBytes + r * 16;
        const uint4 sc = *reinterpret_cast<const uint4 *>(u);
        const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
        const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
        const float dd = __fmul_rn(half_bits_to_float((uint32_t)(A >> 48)),
                                   (float)(uint32_t)((A >> (6 * k)) & 63u));
        const float mm = __fmul_rn(half_bits_to_float((uint32_t)(B >> 48)),
                                   (float)(uint32_t)((B >> (6 * k)) & 63u));
        const uint8_t byte = u[512 * (k + 1) + (j & 15)];
        const float q = (float)(j < 16 ? (byte & 15) : (byte >> 4));
        x[(size_t)row * H + c] = __fadd_rn(__fmul_rn(dd, q), -mm);
    }
}

// ------------------------------------------------------------------ RMSNorm + A8
// sumsq (engine/src/forward_ops.c:170-181): 4 interleaved partial sums over the first n/4*4
// elements, sequential tail, result ((c0 + c1) + (c2 + c3)) + tail. Threads 0..3 of warp 0
// run the four chains, thread 4 the tail.
__device__ float sumsq_ref(const float *x, int n) {
    const int lane = threadIdx.x & 31;
    float c = 0.0f;
    const int n4 = n & ~3;
    if (lane < 4) {
#pragma unroll 32
        for (int i = lane; i < n4; i += 4) c = madd(c, x[i], x[i]);
    } else if (lane == 4) {
        for (int i = n4; i < n; i++) c = madd(c, x[i], x[i]);
    }
    const float c1 = __shfl_sync(0xffffffffu, c, 1), c2 = __shfl_sync(0xffffffffu, c, 2);
    const float c3 = __shfl_sync(0xffffffffu, c, 3), t = __shfl_sync(0xffffffffu, c, 4);
    const float c0 = __shfl_sync(0xffffffffu, c, 0);
    return __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), t);
}

// pf_softmax_exp's sum (forward_ops.c:320-353): 4 interleaved partial sums over the first
// n/4*4 elements, sequential tail, ((c0 + c1) + (c2 + c3)) + tail. Called by warp 0.
__device__ float sum4_ref(const float *a, int n) {
    const int lane = threadIdx.x & 31;
    float c = 0.0f;
    const int n4 = n & ~3;
    if (lane < 4) {
#pragma unroll 32
        for (int i = lane; i < n4; i += 4) c = __fadd_rn(c, a[i]);
    } else if (lane == 4) {
        for (int i = n4; i < n; i++) c = __fadd_rn(c, a[i]);
    }
    const float c1 = __shfl_sync(0xffffffffu, c, 1), c2 = __shfl_sync(0xffffffffu, c, 2);
    const float c3 = __shfl_sync(0xffffffffu, c, 3), t = __shfl_sync(0xffffffffu, c, 4);
    const float c0 = __shfl_sync(0xffffffffu, c, 0);
    return __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), t);
}

// pf_rmsnorm (forward_ops.c:191-200): r = 1 / sqrtf(sumsq / n + eps), y = (x * r) * w, then
// A8 blocks of 32 (kern_quant_act). One CTA per row, H floats of shared memory.
__global__ void k_norm_quant(const float *x, const float *w, int H, float eps, const Step *st,
                             Act out) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.y;   // the sequence (multi-sequence passes)
    if ((int)blockIdx.x >= st->n) return;
    const int v = st->row0 + blockIdx.x;
    extern __shared__ float xs[];   // [H] x, then [H] w
    __shared__ float rr;
    float *ws = xs + H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        xs[i] = x[(size_t)v * H + i];
        ws[i] = w[i];
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const float s = sumsq_ref(xs, H);
        if (threadIdx.x == 0) rr = inv_sqrt_ref(__fadd_rn(__fdiv_rn(s, (float)H), eps));
    }
    __syncthreads();
    const float r = rr;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nb = H >> 5;
    for (int b = warp; b < nb; b += nw) {
        const int i = b * 32 + lane;
        const float y = __fmul_rn(__fmul_rn(xs[i], r), ws[i]);
        quant_block_warp(y, lane, out.q + (size_t)v * out.cols + b * 32,
                         out.d + (size_t)v * nb + b, out.fs + (size_t)v * nb + b);
    }
}

// plain A8 quantisation of n rows (kernel-level C-ABI entry point)
__global__ void k_quant_act(const float *x, int n, int cols, Act out) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nb = cols >> 5;
    if (gw >= n * nb) return;
    const int v = gw / nb, b = gw % nb;
    quant_block_warp(x[(size_t)v * cols + b * 32 + lane], lane,
                     out.q + (size_t)v * cols + b * 32, out.d + (size_t)v * nb + b,
                     out.fs + (size_t)v * nb + b);
}

// ------------------------------------------------------------------ Gated DeltaNet layer
// pf_linear_attn (engine/src/forward_lin.c:322-361) after its four projections, which the
// W_in matvec already wrote to y[t][0..ldy): qkv | z | b | a.
//  1. pending conv commit of the last verify pass (pf_lin_commit, :413-432), then causal
//     depthwise conv + SiLU per channel and token (pre_task :264-286, pf_conv_silu
//     forward_ops.c:237-260); a logged pass shifts the live state by token 0 only and records
//     the raw inputs of rows 1..;
//  2. L2 norm of q and k per head (pf_l2norm_scale, forward_ops.c:202-210), q scaled by
//     1/sqrt(dk);
//  3. gates: beta = 1 / (1 + expf(-b)), decay = expf(A * softplus(a + dt_bias)) with glibc's
//     expf / log1pf values (:19, :288-293);
//  4. the recurrence (delta_rule / pf_lin_rule / replay_first: matvec_ref.c:114-188,
//     kern_lin.c:42-62): first the deferred updates of the last commit, then per token
//     S *= decay; kv = S^T k; delta = (v - kv) beta; S += k delta^T; o = S^T q, no fused
//     multiply-add, sums over the key index in order; token 0 in place, rows 1.. of a logged
//     pass on the register copy with k | delta | decay logged;
//  5. gated RMSNorm rmsnorm(o) * w * silu(z) (post_task :298-309);
//  6. A8 quantisation of the result for out_proj.
// One CTA per key head (rep value heads of 128 columns each); thread (r, j) keeps column j of
// value head r's 128 x 128 state in registers.
constexpr int kDK = 128, kDV = 128;

struct DnSmem {   // carved from dynamic shared memory
    float *cq, *ck, *cv, *so;  // [nmax][dk], [nmax][dk], [nmax][rep*dv], [nmax][rep*dv]
    float *beta, *decay;       // [nmax][rep]
    float *kp;                 // [rep][dk] replay staging
    float *pdec;               // [rep]
    float *rn;                 // [nmax][rep] gated-norm factors
};

__global__ void __launch_bounds__(128, 1) k_deltanet(LinLayer L, LinDims d, const float *y, Step *st,
                                                  Act out) {
    pdl_wait();
    pdl_trigger();
    const int n = st->n;
    if (n <= 0) return;
    const int logged = st->logged, pend_keep = st->pend_keep, pend_conv = st->pend_conv;
    const int wr = st->wr;
    const int kh = blockIdx.x, rep = d.rep, tid = threadIdx.x, nthr = blockDim.x;
    extern __shared__ __align__(16) float dsm[];
    DnSmem s;
    s.cq = dsm;
    s.ck = s.cq + kMaxRows * kDK;
    s.cv = s.ck + kMaxRows * kDK;
    s.so = s.cv + kMaxRows * rep * kDV;
    s.beta = s.so + kMaxRows * rep * kDV;
    s.decay = s.beta + kMaxRows * rep;
    s.kp = s.decay + kMaxRows * rep;
    s.pdec = s.kp + kMaxRows * kDK;
    s.rn = s.pdec + kMaxRows;
    const int C = d.C, K = d.K, S = K - 1;

    // ---- 0. start the recurrent state load (registers) and the replay-log staging: neither
    //         depends on this pass's activations, so they overlap the conv / norm / gate work
    float Sc[kDK];
    const bool preload = rep == 1;
    const int j = tid;
    if (preload) {
        const float *rec0 = L.rec + (size_t)(kh * rep) * kDK * kDV + j;
#pragma unroll
        for (int i = 0; i < kDK; i++) Sc[i] = rec0[(size_t)i * kDV];
    }
    // ---- 1a. gates (only need b and a)
    for (int u = tid; u < n * rep; u += nthr) {
        const int t = u / rep, r = u % rep, h = kh * rep + r;
        const float b = y[(size_t)t * d.ldy + C + d.vd + h];
        const float a = y[(size_t)t * d.ldy + C + d.vd + d.nv + h];
        s.beta[t * rep + r] = __fdiv_rn(1.0f, __fadd_rn(1.0f, glibc_expf(-b)));
        const float xs = __fadd_rn(a, L.dt_bias[h]);
        const float sp = xs > 20.0f ? xs : glibc_log1pf(glibc_expf(xs));
        s.decay[t * rep + r] = glibc_expf(__fmul_rn(L.A[h], sp));
    }

    // ---- 1. conv + SiLU
    const int nch = 2 * kDK + rep * kDV;
    for (int ch = tid; ch < nch; ch += nthr) {
        int c;
        float *dst;
        int dstride;
        if (ch < kDK) { c = kh * kDK + ch; dst = s.cq + ch; dstride = kDK; }
        else if (ch < 2 * kDK) { c = d.kd + kh * kDK + (ch - kDK); dst = s.ck + (ch - kDK); dstride = kDK; }
        else {
            const int vv = ch - 2 * kDK;
            c = 2 * d.kd + kh * rep * kDV + vv;
            dst = s.cv + vv;
            dstride = rep * kDV;
        }
        float stt[8], wc[8], live[8];
        for (int j = 0; j < S; j++) stt[j] = L.conv_state[(size_t)j * C + c];
        for (int j = 0; j < K; j++) wc[j] = L.conv_w[(size_t)c * K + j];
        if (pend_conv > 1) {   // new state = last S rows of [state after token 0, inputs 1..e-1]
            const int e1 = pend_conv - 1;
            float ns[8];
            for (int j = 0; j < S; j++) {
                const int src = j + e1;
                ns[j] = src < S ? stt[src] : L.xin[(size_t)(src - S + 1) * C + c];
            }
            for (int j = 0; j < S; j++) stt[j] = ns[j];
        }
        for (int t = 0; t < n; t++) {
            const float xc = y[(size_t)t * d.ldy + c];
            float acc = __fmul_rn(wc[0], S > 0 ? stt[0] : xc);
            for (int j = 1; j < K; j++) acc = madd(acc, wc[j], j < S ? stt[j] : xc);
            for (int j = 0; j + 1 < S; j++) stt[j] = stt[j + 1];
            if (S > 0) stt[S - 1] = xc;
            dst[t * dstride] = pf_silu(acc);
            if (logged) {
                if (t == 0) for (int j = 0; j < S; j++) live[j] = stt[j];
                else L.xin[(size_t)t * C + c] = xc;
            }
        }
        const float *fin = logged ? live : stt;
        for (int j = 0; j < S; j++) L.conv_state[(size_t)j * C + c] = fin[j];
    }
    __syncthreads();

    // ---- 2. L2 norm of q and k, 4 lanes per (token, vector)
    {
        const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
        const float qscale = inv_sqrt_ref((float)kDK);
        for (int u0 = warp * 8; u0 < 2 * n; u0 += nw * 8) {
            const int u = u0 + (lane >> 2), l = lane & 3;
            const bool act = u < 2 * n;
            float *vec = act ? ((u & 1) ? s.ck : s.cq) + (u >> 1) * kDK : s.cq;
            float c = 0.0f;
            if (act) {
#pragma unroll 32
                for (int i = l; i < kDK; i += 4) c = madd(c, vec[i], vec[i]);
            }
            const int base = lane & ~3;
            const float c0 = __shfl_sync(0xffffffffu, c, base), c1 = __shfl_sync(0xffffffffu, c, base + 1);
            const float c2 = __shfl_sync(0xffffffffu, c, base + 2), c3 = __shfl_sync(0xffffffffu, c, base + 3);
            const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
            const float r = inv_sqrt_ref(__fadd_rn(ss, 1e-6f));
            __syncwarp();
            if (act) {
                const float sc = (u & 1) ? 1.0f : qscale;
                for (int i = l; i < kDK; i += 4) vec[i] = __fmul_rn(__fmul_rn(vec[i], r), sc);
            }
        }
    }
    __syncthreads();
    // ---- 4. recurrence, value heads of this key head one after another
    const size_t logw = (size_t)kDK + kDV + 1;
    for (int r = 0; r < rep; r++) {
        const int h = kh * rep + r;
        float *rec = L.rec + (size_t)h * kDK * kDV + j;
        if (!preload) {
#pragma unroll
            for (int i = 0; i < kDK; i++) Sc[i] = rec[(size_t)i * kDV];
        }
        if (pend_keep > 0) {   // deferred commit: rows 1..keep of half wr^1 (<= kMaxRows - 1)
            float dl[kMaxRows];
            __syncthreads();
            for (int tp = 1; tp <= pend_keep; tp++) {
                const float *u = L.upd + (((size_t)(wr ^ 1) * d.cap + tp) * d.nv + h) * logw;
                s.kp[(tp - 1) * kDK + j] = u[j];
                dl[tp - 1] = u[kDK + j];
                if (j == 0) s.pdec[tp - 1] = u[kDK + kDV];
            }
            __syncthreads();
            for (int tp = 0; tp < pend_keep; tp++) {
                const float pd = s.pdec[tp], dv_ = dl[tp];
                const float *kr = s.kp + tp * kDK;
#pragma unroll
                for (int i = 0; i < kDK; i++)
                    Sc[i] = __fadd_rn(__fmul_rn(Sc[i], pd), __fmul_rn(kr[i], dv_));
            }
        }
        for (int t = 0; t < n; t++) {
            const float *qt = s.cq + t * kDK, *kt = s.ck + t * kDK;
            const float dec = s.decay[t * rep + r], beta = s.beta[t * rep + r];
            float kv = 0.0f;
#pragma unroll
            for (int i = 0; i < kDK; i++) {
                Sc[i] = __fmul_rn(Sc[i], dec);
                kv = madd(kv, Sc[i], kt[i]);
            }
            const float delta = __fmul_rn(__fadd_rn(s.cv[t * rep * kDV + r * kDV + j], -kv), beta);
            float o = 0.0f;
#pragma unroll
            for (int i = 0; i < kDK; i++) {
                Sc[i] = __fadd_rn(Sc[i], __fmul_rn(kt[i], delta));
                o = madd(o, Sc[i], qt[i]);
            }
            s.so[t * rep * kDV + r * kDV + j] = o;
            if (logged) {
                if (t == 0) {
#pragma unroll
                    for (int i = 0; i < kDK; i++) rec[(size_t)i * kDV] = Sc[i];
                } else {
                    float *u = L.upd + (((size_t)wr * d.cap + t) * d.nv + h) * logw;
                    u[kDK + j] = delta;
                    u[j] = kt[j];
                    if (j == 0) u[kDK + kDV] = dec;
                }
            }
        }
        if (!logged) {
#pragma unroll
            for (int i = 0; i < kDK; i++) rec[(size_t)i * kDV] = Sc[i];
        }
    }
    __syncthreads();

    // ---- 5. gated RMSNorm: per (token, head) r = 1 / sqrtf(sumsq(o) / dv + eps), 4 chains
    {
        const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
        for (int u0 = warp * 8; u0 < n * rep; u0 += nw * 8) {
            const int u = u0 + (lane >> 2), l = lane & 3;
            const bool act = u < n * rep;
            const float *vec = act ? s.so + (size_t)(u / rep) * rep * kDV + (u % rep) * kDV : s.so;
            float c = 0.0f;
            if (act)
                for (int i = l; i < kDV; i += 4) c = madd(c, vec[i], vec[i]);
            const int base = lane & ~3;
            const float c0 = __shfl_sync(0xffffffffu, c, base), c1 = __shfl_sync(0xffffffffu, c, base + 1);
            const float c2 = __shfl_sync(0xffffffffu, c, base + 2), c3 = __shfl_sync(0xffffffffu, c, base + 3);
            const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
            if (act && l == 0) s.rn[u] = inv_sqrt_ref(__fadd_rn(__fdiv_rn(ss, (float)kDV), d.eps));
        }
    }
    __syncthreads();
    // ---- 6. y = (o * r) * w * silu(z), A8 per 32 columns
    {
        const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
        const int nblk = n * rep * (kDV / 32);
        const int nbo = out.cols >> 5;
        for (int b = warp; b < nblk; b += nw) {
            const int t = b / (rep * (kDV / 32)), rem = b % (rep * (kDV / 32));
            const int rr = rem / (kDV / 32), cb = rem % (kDV / 32);
            const int jj = cb * 32 + lane, hh = kh * rep + rr;
            const float rn = s.rn[t * rep + rr];
            float v = __fmul_rn(__fmul_rn(s.so[t * rep * kDV + rr * kDV + jj], rn), L.norm_w[jj]);
            const float z = y[(size_t)t * d.ldy + C + hh * kDV + jj];
            v = __fmul_rn(v, pf_silu(z));
            const int col = hh * kDV + jj;
            quant_block_warp(v, lane, out.q + (size_t)t * out.cols + (col & ~31),
                             out.d + (size_t)t * nbo + (col >> 5), out.fs + (size_t)t * nbo + (col >> 5));
        }
    }
}

// Apply every deferred commit now (pf_lin_flush, engine/src/forward_lin.c:435-444, and the
// conv half of pf_lin_commit): grid (key heads, linear layers).
struct FlushArgs {
    LinLayer layers[kMaxLayers];
};

__global__ void k_flush(FlushArgs fa, LinDims d, const Step *st) {
    pdl_wait();
    pdl_trigger();
    const int seq = blockIdx.z;   // the sequence (multi-sequence batches)
    st += seq;
    const int keep = st->pend_keep, pend_conv = st->pend_conv, wr = st->wr;
    LinLayer L = fa.layers[blockIdx.y];
    L.conv_state += seq * d.ss_conv;
    L.rec += seq * d.ss_rec;
    L.xin += seq * d.ss_xin;
    L.upd += seq * d.ss_upd;
    const int kh = blockIdx.x, rep = d.rep, tid = threadIdx.x, nthr = blockDim.x;
    const int C = d.C, S = d.K - 1;
    if (pend_conv > 1) {
        const int nch = 2 * kDK + rep * kDV, e1 = pend_conv - 1;
        for (int ch = tid; ch < nch; ch += nthr) {
            int c;
            if (ch < kDK) c = kh * kDK + ch;
            else if (ch < 2 * kDK) c = d.kd + kh * kDK + (ch - kDK);
            else c = 2 * d.kd + kh * rep * kDV + (ch - 2 * kDK);
            float stt[8], ns[8];
            for (int j = 0; j < S; j++) stt[j] = L.conv_state[(size_t)j * C + c];
            for (int j = 0; j < S; j++) {
                const int src = j + e1;
                ns[j] = src < S ? stt[src] : L.xin[(size_t)(src - S + 1) * C + c];
            }
            for (int j = 0; j < S; j++) L.conv_state[(size_t)j * C + c] = ns[j];
        }
    }
    if (keep > 0) {
        const int j = tid;
        const size_t logw = (size_t)kDK + kDV + 1;
        for (int r = 0; r < rep; r++) {
            const int h = kh * rep + r;
            float *rec = L.rec + (size_t)h * kDK * kDV + j;
            for (int tp = 1; tp <= keep; tp++) {
                const float *u = L.upd + (((size_t)(wr ^ 1) * d.cap + tp) * d.nv + h) * logw;
                const float pd = u[kDK + kDV], dl = u[kDK + j];
                for (int i = 0; i < kDK; i++)   // pf_lin_apply: row *= decay; row += k_i * delta_j
                    rec[(size_t)i * kDV] = __fadd_rn(__fmul_rn(rec[(size_t)i * kDV], pd), __fmul_rn(u[i], dl));
            }
        }
    }
}

// End of a pass: its deferred commit has been consumed by every layer.
__global__ void k_pass_end(Step *st) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.x;   // the sequence (multi-sequence passes)
    if (st->n <= 0) return;   // no pass ran (generation finished): the commit is still owed
    st->pend_keep = 0;
    st->pend_conv = 0;
}

__global__ void k_clear_pending(Step *st) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.x;   // the sequence (multi-sequence batches)
    st->pend_keep = 0;
    st->pend_conv = 0;
}

// Host-chosen shapes of a multi-sequence pass, one CTA per sequence.
__global__ void k_set_pass_seqs(Step *st, const SeqPass *ps) {
    pdl_wait();
    pdl_trigger();
    const SeqPass &p = ps[blockIdx.x];
    st += blockIdx.x;
    if (threadIdx.x == 0) {
        st->n = p.n;
        st->pos0 = p.pos0;
        st->row0 = p.row0;
        st->logged = p.logged;
    }
    if ((int)threadIdx.x < p.n && threadIdx.x < kMaxRows) st->tokens[threadIdx.x] = p.tokens[threadIdx.x];
}

// Sequences of a batch whose generation has finished.
__global__ void k_count_done(const Step *st, int nseq, int *ndone) {
    pdl_wait();
    pdl_trigger();
    int c = 0;
    for (int i = threadIdx.x; i < nseq; i += blockDim.x) c += st[i].done ? 1 : 0;
    c = warp_sum_int(c);
    __shared__ int part[32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += part[w];
        *ndone = t;
    }
}

// Host-chosen pass (prefill chunks, plain eval): shape and tokens by value.
struct PassArgs {
    int n, pos0, logged;
    int tokens[kMaxRows];
};
__global__ void k_set_pass(Step *st, PassArgs a) {
    pdl_wait();
    pdl_trigger();
    st->n = a.n;
    st->pos0 = a.pos0;
    st->logged = a.logged;
    for (int i = 0; i < a.n && i < kMaxRows; i++) st->tokens[i] = a.tokens[i];
}

// Generation parameters before k_gen_start.
// blockIdx.x: the sequence of a batch, whose drafter seed is seeds[seq] when seeds is given.
__global__ void k_set_gen(Step *st, GenArgs g, const unsigned long long *seeds) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.x;
    if (seeds) g.seed = seeds[blockIdx.x];
    st->n_max = g.n_max;
    st->k = g.k;
    st->eos = g.eos;
    st->n_stop = g.n_stop;
    for (int i = 0; i < 8; i++) st->stop_ids[i] = g.stop_ids[i];
    st->max_ctx = g.max_ctx;
    st->vocab = g.vocab;
    st->p24 = g.p24;
    st->seed = g.seed;
    st->rounds = st->drafted = st->accepted = 0;
    st->count = 0;
    st->done = 0;
    st->status = 0;
    st->drafter = g.drafter;
    st->ngram = g.ngram;
    st->use_ng = 0;
    st->ng_rounds = st->ng_drafted = st->ng_accepted = 0;
    st->adaptive = g.adaptive;   // pf_adapt_init (spec_adapt.c): measurements cleared
    st->chain_stop = 0;
    st->conf = 0.0f;
    for (int i = 0; i <= kMaxRows; i++) st->ad_tv[i] = 0.0;
    st->ad_t_plain = st->ad_r_tok = st->ad_r_sec = 0.0;
    st->ad_n_spec = st->ad_plain_mode = st->ad_plain_run = st->ad_probing = 0;
    st->ad_probe_after = 8;
    st->last_e = 0;
}

// ------------------------------------------------------------------ attention
// pf_full_attn (engine/src/forward_attn.c:231-266), first part: per token, the K row of each
// KV head (RMSNorm with k_norm, RoPE, stored at position pos0 + t), its V row, and every query
// head (RMSNorm with q_norm, RoPE). RoPE tables come from the host, computed with glibc
// exactly as pf_rope_tables does (forward.c:19-32). grid (rows, nq + nkv), hd threads.
// A K or V row at the storage precision of pf_kv_store (forward_kv.c:83-123), widened back to
// fp32 as pf_kv_widen reads it (forward_kv.c:139-166), one element per thread of the block:
// fp16 rounds to nearest even (widening is exact); int8 scales by the row's absolute maximum
// (exact in any order), q = rint(x * (127 / amax)) clamped to [-127, 127] (NaN: 0), value
// q * (amax / 127). The attention kernels then read fp32 rows equal to the reference's widened
// rows. Every thread of the block calls it (block-wide maximum).
__device__ float kv_store_round(float x, int dtype, float *scale_out, float *red) {
    if (dtype == PINFER_KV_F16) return __half2float(__float2half_rn(x));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float a = fabsf(x);
    for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) red[warp] = a;
    __syncthreads();
    if (warp == 0) {
        a = lane < nw ? red[lane] : 0.0f;
        for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) red[32] = a;
    }
    __syncthreads();
    const float amax = red[32];
    __syncthreads();   // red is free again
    const float inv = amax > __fdiv_rn(127.0f, FLT_MAX) ? __fdiv_rn(127.0f, amax) : 0.0f;
    const float sc = __fdiv_rn(amax, 127.0f);
    const float yq = rintf(__fmul_rn(x, inv));
    const int q = yq > 127.0f ? 127 : yq < -127.0f ? -127 : (yq == yq ? (int)yq : 0);
    *scale_out = sc;
    return __fmul_rn((float)q, sc);
}

__global__ void k_attn_prep(AttnLayer L, AttnDims d, const float *y, float *qbuf,
                            const Step *st) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x % d.rps, seq = blockIdx.x / d.rps;   // row t of sequence seq
    st += seq;
    if (t >= st->n) return;
    const int idx = blockIdx.y, hd = d.hd, tid = threadIdx.x;
    const int pos = st->pos0 + t;
    if (pos >= d.max_ctx) return;
    const int row = st->row0 + t;
    L.kc += seq * d.ss_kv;
    L.vc += seq * d.ss_kv;
    extern __shared__ float xa[];
    __shared__ float rr;
    const float *src;
    const float *w;
    if (idx < d.nq) { src = y + (size_t)row * d.ldy + (size_t)2 * hd * idx; w = L.q_norm; }
    else { src = y + (size_t)row * d.ldy + (size_t)2 * hd * d.nq + (size_t)(idx - d.nq) * hd; w = L.k_norm; }
    xa[tid] = src[tid];
    __syncthreads();
    if (tid < 32) {
        const float sq = sumsq_ref(xa, hd);
        if (tid == 0) rr = inv_sqrt_ref(__fadd_rn(__fdiv_rn(sq, (float)hd), d.eps));
    }
    __syncthreads();
    float v = __fmul_rn(__fmul_rn(xa[tid], rr), w[tid]);
    __syncthreads();
    xa[tid] = v;
    __syncthreads();
    const int h2 = d.rot >> 1;
    if (tid < h2) {   // pf_rope (forward_ops.c:149-165): pairs (i, i + rot/2)
        const float c = d.rope_cos[(size_t)pos * h2 + tid], sn = d.rope_sin[(size_t)pos * h2 + tid];
        const float a = xa[tid], b = xa[tid + h2];
        v = __fadd_rn(__fmul_rn(a, c), -__fmul_rn(b, sn));
    } else if (tid < 2 * h2) {
        const int i = tid - h2;
        const float c = d.rope_cos[(size_t)pos * h2 + i], sn = d.rope_sin[(size_t)pos * h2 + i];
        const float a = xa[i], b = xa[tid];
        v = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
    }
    if (idx < d.nq) {
        qbuf[((size_t)row * d.nq + idx) * hd + tid] = v;
    } else {
        const int g = idx - d.nq;
        const size_t r = (size_t)g * d.max_ctx + pos;
        float vv = y[(size_t)row * d.ldy + (size_t)2 * hd * d.nq + (size_t)d.nkv * hd + (size_t)g * hd + tid];
        if (d.kv_dtype != PINFER_KV_F32) {   // uniform over the block
            __shared__ float red[33];
            float sk = 0.0f, sv = 0.0f;
            v = kv_store_round(v, d.kv_dtype, &sk, red);
            vv = kv_store_round(vv, d.kv_dtype, &sv, red);
            if (d.kv_dtype == PINFER_KV_I8 && tid == 0 && L.ks) {
                L.ks[r] = sk;
                L.vs[r] = sv;
            }
        }
        L.kc[r * hd + tid] = v;
        L.vc[r * hd + tid] = vv;
    }
}

// Second part (attend / score_task / softmax_task / pv_task, forward_attn.c:95-229): per
// (token, query head): scores pf_dot(q, K row) * (1/sqrt(hd)) with pf_dot's 16-lane order
// (forward_ops.c:265-287), softmax max, pf_expf(a - max) and the 4-lane sum
// (forward_ops.c:320-353), p = a * (1 / sum), P.V accumulated in row order from zero,
// o *= sigmoid(gate), then A8 blocks of 32 for o_proj. grid (rows, nq), hd threads,
// dynamic shared memory: q [hd] + att [max_ctx].
__global__ void k_attn(AttnLayer L, AttnDims d, const float *y, const float *qbuf,
                       const Step *st, Act out) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= st->n) return;
    const int h = blockIdx.y, hd = d.hd, tid = threadIdx.x;
    const int g = h / (d.nq / d.nkv);
    const int pos = st->pos0 + t;
    if (pos >= d.max_ctx) return;
    const int np = pos + 1;
    extern __shared__ float sm[];
    float *q = sm, *att = sm + hd;
    __shared__ float red[32];
    __shared__ float s_mx, s_inv;
    q[tid] = qbuf[((size_t)t * d.nq + h) * hd + tid];
    __syncthreads();
    const float scale = inv_sqrt_ref((float)hd);
    const int lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const float *K = L.kc + (size_t)g * d.max_ctx * hd;
    for (int p0 = warp * 2; p0 < np; p0 += nw * 2) {
        const int p = p0 + (lane >> 4), l = lane & 15;
        float c = 0.0f;
        if (p < np) {
            const float *kr = K + (size_t)p * hd;
            for (int i = l; i < hd; i += 16) c = madd(c, q[i], kr[i]);
        }
        c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 1));
        c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 2));
        c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 4));
        c = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 8));
        if (l == 0 && p < np) att[p] = __fmul_rn(__fadd_rn(c, 0.0f), scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int p = tid; p < np; p += blockDim.x) m = fmaxf(m, att[p]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid < 32) {
        float mm = tid < nw ? red[tid] : -INFINITY;
        for (int o = 16; o; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        if (tid == 0) s_mx = mm;
    }
    __syncthreads();
    const float mx = s_mx;
    for (int p = tid; p < np; p += blockDim.x) att[p] = pf_expf(__fadd_rn(att[p], -mx));
    __syncthreads();
    if (tid < 32) {
        const float sum = sum4_ref(att, np);
        if (tid == 0) s_inv = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int p = tid; p < np; p += blockDim.x) att[p] = __fmul_rn(att[p], inv);
    __syncthreads();
    const float *V = L.vc + (size_t)g * d.max_ctx * hd + tid;
    float o = 0.0f;
    int jj = 0;
    for (; jj + 8 <= np; jj += 8) {
        float vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) vv[u] = V[(size_t)(jj + u) * hd];
#pragma unroll
        for (int u = 0; u < 8; u++) o = madd(o, att[jj + u], vv[u]);
    }
    for (; jj < np; jj++) o = madd(o, att[jj], V[(size_t)jj * hd]);
    const float gate = y[(size_t)t * d.ldy + (size_t)2 * hd * h + hd + tid];
    o = __fmul_rn(o, pf_sigmoid(gate));
    const int col = h * hd + tid, nbo = out.cols >> 5;
    quant_block_warp(o, lane, out.q + (size_t)t * out.cols + (col & ~31),
                     out.d + (size_t)t * nbo + (col >> 5), out.fs + (size_t)t * nbo + (col >> 5));
}


// Second part of the attention (attend / score_task / softmax_task / pv_task,
// forward_attn.c:95-229), per (token, query head), hd threads:
//  scores   pf_dot(q, K row) * (1/sqrt(hd)): each thread keeps pf_dot's 16 interleaved partial
//           sums of one position in registers (forward_ops.c:265-287), K rows read as float4;
//  softmax  max, pf_expf(a - max), the 4-lane sum (forward_ops.c:320-353), p = a * (1/sum);
//  P.V      row order from zero, per column; V rows stream into a per-thread cp.async ring in
//           shared memory (`ring` rows in flight), so the sequential chain reads on-chip data;
//  o *= sigmoid(gate), then A8 blocks of 32 for o_proj.

constexpr int kAttnHd = 256;
constexpr int kVRing = 96;
constexpr int kVGroup = 8;

__global__ void __launch_bounds__(kAttnHd) k_attn2(AttnLayer L, AttnDims d, const float *y,
                                                   const float *qbuf, const Step *st, Act out) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= st->n) return;
    constexpr int HD = kAttnHd;
    const int h = blockIdx.y, tid = threadIdx.x;
    const int g = h / (d.nq / d.nkv);
    const int pos = st->pos0 + t;
    if (pos >= d.max_ctx) return;
    const int np = pos + 1;
    extern __shared__ __align__(16) float asm_[];
    float *q = asm_, *att = asm_ + HD, *vring = att + ((d.max_ctx + 3) & ~3);
    __shared__ float red[32];
    __shared__ float s_mx, s_inv;
    const float *V = L.vc + (size_t)g * d.max_ctx * HD + tid;
    // start the V stream right away (groups of kVGroup rows): it does not depend on the scores
    const int ngroups = (np + kVGroup - 1) / kVGroup;
    for (int gi = 0; gi < kVRing / kVGroup; gi++) {
        for (int r = 0; r < kVGroup; r++) {
            const int j = gi * kVGroup + r;
            if (j < np) cp_async4(vring + (size_t)j * HD + tid, V + (size_t)j * HD);
        }
        cp_async_commit();
    }
    q[tid] = qbuf[((size_t)t * d.nq + h) * HD + tid];
    __syncthreads();
    const float scale = inv_sqrt_ref((float)HD);
    const float *K = L.kc + (size_t)g * d.max_ctx * HD;
    const float4 *q4 = reinterpret_cast<const float4 *>(q);
    for (int p = tid; p < np; p += HD) {
        const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)p * HD);
        float c[16];
#pragma unroll
        for (int l = 0; l < 16; l++) c[l] = 0.0f;
#pragma unroll 4
        for (int i = 0; i < HD / 16; i++) {
            const float4 k0 = __ldg(kr + 4 * i), k1 = __ldg(kr + 4 * i + 1);
            const float4 k2 = __ldg(kr + 4 * i + 2), k3 = __ldg(kr + 4 * i + 3);
            const float4 a0 = q4[4 * i], a1 = q4[4 * i + 1], a2 = q4[4 * i + 2], a3 = q4[4 * i + 3];
            c[0] = madd(c[0], a0.x, k0.x); c[1] = madd(c[1], a0.y, k0.y);
            c[2] = madd(c[2], a0.z, k0.z); c[3] = madd(c[3], a0.w, k0.w);
            c[4] = madd(c[4], a1.x, k1.x); c[5] = madd(c[5], a1.y, k1.y);
            c[6] = madd(c[6], a1.z, k1.z); c[7] = madd(c[7], a1.w, k1.w);
            c[8] = madd(c[8], a2.x, k2.x); c[9] = madd(c[9], a2.y, k2.y);
            c[10] = madd(c[10], a2.z, k2.z); c[11] = madd(c[11], a2.w, k2.w);
            c[12] = madd(c[12], a3.x, k3.x); c[13] = madd(c[13], a3.y, k3.y);
            c[14] = madd(c[14], a3.z, k3.z); c[15] = madd(c[15], a3.w, k3.w);
        }
        float hh[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            hh[k] = __fadd_rn(__fadd_rn(c[4 * k], c[4 * k + 1]), __fadd_rn(c[4 * k + 2], c[4 * k + 3]));
        const float s = __fadd_rn(__fadd_rn(hh[0], hh[1]), __fadd_rn(hh[2], hh[3]));
        att[p] = __fmul_rn(__fadd_rn(s, 0.0f), scale);
    }
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5, nw = HD >> 5;
    float m = -INFINITY;
    for (int p = tid; p < np; p += HD) m = fmaxf(m, att[p]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid < 32) {
        float mm = tid < nw ? red[tid] : -INFINITY;
        for (int o = 16; o; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        if (tid == 0) s_mx = mm;
    }
    __syncthreads();
    const float mx = s_mx;
    for (int p = tid; p < np; p += HD) att[p] = pf_expf(__fadd_rn(att[p], -mx));
    __syncthreads();
    if (tid < 32) {
        const float sum = sum4_ref(att, np);
        if (tid == 0) s_inv = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int p = tid; p < np; p += HD) att[p] = __fmul_rn(att[p], inv);
    __syncthreads();
    float o = 0.0f;
    for (int gi = 0; gi < ngroups; gi++) {
        cp_async_wait<kVRing / kVGroup - 1>();
        const int j0 = gi * kVGroup;
        float *slot = vring + (size_t)(j0 % kVRing) * HD + tid;
        float v[kVGroup];
#pragma unroll
        for (int r = 0; r < kVGroup; r++) v[r] = slot[(size_t)r * HD];
#pragma unroll
        for (int r = 0; r < kVGroup; r++)
            if (j0 + r < np) o = madd(o, att[j0 + r], v[r]);
        const int jn = j0 + kVRing;
#pragma unroll
        for (int r = 0; r < kVGroup; r++)
            if (jn + r < np) cp_async4(slot + (size_t)r * HD, V + (size_t)(jn + r) * HD);
        cp_async_commit();
    }
    cp_async_wait<0>();
    const float gate = y[(size_t)t * d.ldy + (size_t)2 * HD * h + HD + tid];
    o = __fmul_rn(o, pf_sigmoid(gate));
    const int col = h * HD + tid, nbo = out.cols >> 5;
    quant_block_warp(o, lane, out.q + (size_t)t * out.cols + (col & ~31),
                     out.d + (size_t)t * nbo + (col >> 5), out.fs + (size_t)t * nbo + (col >> 5));
}

size_t attn2_smem(int max_ctx) {
    return sizeof(float) * ((size_t)kAttnHd + ((max_ctx + 3) & ~3) + (size_t)kVRing * kAttnHd);
}

// ------------------------------------------------------------------ attention, one cluster per (token, head)
// The same arithmetic as k_attn2 spread over a thread-block cluster of kAttnCL CTAs, so that one
// (token, head) pair draws on kAttnCL SMs' L2 bandwidth instead of one:
//   1. CTA c scores the positions of its slice [c per, (c + 1) per): 4 lanes per position, lane
//      k4 holding the pf_dot partial sums 4 k4 .. 4 k4 + 3 (element 16 i + l feeds sum l), the
//      tree of partial sums finished with quad shuffles (IEEE addition commutes, so every lane
//      of the quad forms the identical value). Meanwhile CTA c's 32 output columns of V
//      (rows 0..np-1) stream into its shared memory with cp.async.
//   2. cluster barrier; every CTA gathers the np scores from the cluster's shared memory
//      (distributed shared memory loads) and runs the reference softmax on its own copy:
//      fmaxf max, pf_expf, sum4_ref, one division, scaling (identical code to k_attn2);
//   3. warp 0 runs the ordered PV chain o += att[p] * V[p][col] for its 32 columns, gates it
//      and A8-quantises the 32-column block (one block per CTA).
// The whole cluster leaves together: t and pos are uniform over it, and every CTA waits on the
// cluster barrier before exit so no peer reads shared memory that is gone.
constexpr int kAttnCL = 8;
constexpr int kAttnSlice = kAttnHd / kAttnCL;   // 32 output columns per CTA
constexpr int kAttnChunk = 32;                   // V rows per cp.async group (one 16 B copy per thread)
constexpr int kAttnRing = 16;                    // chunks in the V ring (512 rows, 64 KB)

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// a float of CTA `rank`'s shared memory at the offset of `local` in this CTA's
__device__ __forceinline__ float ld_dsmem(const float *local, uint32_t rank) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}

size_t attn3_smem(int max_ctx) {
    const size_t per = ((size_t)max_ctx + kAttnCL - 1) / kAttnCL;
    return sizeof(float) * ((size_t)kAttnHd + ((per + 3) & ~(size_t)3) + (((size_t)max_ctx + 3) & ~(size_t)3) +
                            (size_t)kAttnRing * kAttnChunk * kAttnSlice);
}

__global__ void __cluster_dims__(kAttnCL, 1, 1) __launch_bounds__(kAttnHd)
    k_attn3(AttnLayer L, AttnDims d, const float *y, const float *qbuf, const Step *st, Act out) {
    pdl_wait();
    pdl_trigger();
    constexpr int HD = kAttnHd;
    const int t = blockIdx.z % d.rps, seq = blockIdx.z / d.rps, h = blockIdx.y, tid = threadIdx.x;
    st += seq;                              // row t of sequence seq (multi-sequence passes)
    if (t >= st->n) return;                 // uniform over the cluster
    const int pos = st->pos0 + t;
    if (pos >= d.max_ctx) return;           // uniform over the cluster
    const int row = st->row0 + t;
    L.kc += seq * d.ss_kv;
    L.vc += seq * d.ss_kv;
    const uint32_t c = cluster_rank();
    const int np = pos + 1, g = h / (d.nq / d.nkv);
    const int per = (d.max_ctx + kAttnCL - 1) / kAttnCL;
    extern __shared__ __align__(16) float asm3[];
    float *q = asm3, *part = q + HD, *att = part + ((per + 3) & ~3);
    float *vs = att + ((d.max_ctx + 3) & ~3);   // V ring: [kAttnRing][kAttnChunk rows][32]
    __shared__ float red[32];
    __shared__ float s_mx, s_inv;

    // V columns c*32 .. c*32+31 stream through a ring of kAttnRing chunks of kAttnChunk rows
    // (8 x 16 bytes per row). The first kAttnRing - 1 chunks start now, behind the scores, one
    // copy per thread per chunk; the CTA waits for them once, before the P.V chain. The chain
    // and the later chunks are warp 0's: lane l copies row l of a chunk, one cp.async group per
    // chunk, so the chain waits on its own copies and a warp barrier only.
    const float *V = L.vc + (size_t)g * d.max_ctx * HD + c * kAttnSlice;
    const int nch = (np + kAttnChunk - 1) / kAttnChunk;
    const int lane = tid & 31, warp = tid >> 5, nw = HD >> 5;
    static_assert(kAttnChunk * 8 == kAttnHd, "one 16-byte copy per thread per chunk");
    for (int ch = 0; ch < kAttnRing - 1 && ch < nch; ch++) {
        const int r = ch * kAttnChunk + (tid >> 3), k = tid & 7;
        if (r < np)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                         ::"r"(smem_u32(vs + ((size_t)ch * kAttnChunk + (tid >> 3)) * kAttnSlice + 4 * k)),
                         "l"(V + (size_t)r * HD + 4 * k) : "memory");
    }
    cp_async_commit();
    auto issue_chunk = [&](int ch) {
        const int r = ch * kAttnChunk + lane;
        if (ch < nch && r < np) {
            const uint32_t dst = smem_u32(vs + ((size_t)(ch % kAttnRing) * kAttnChunk + lane) * kAttnSlice);
#pragma unroll
            for (int k = 0; k < 8; k++)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 16 * k), "l"(V + (size_t)r * HD + 4 * k)
                             : "memory");
        }
        cp_async_commit();   // one group per chunk, empty past the end
    };
    static_assert(kAttnChunk == 32, "one row per lane per chunk");
    q[tid] = qbuf[((size_t)row * d.nq + h) * HD + tid];
    const float gate = tid < kAttnSlice ? y[(size_t)row * d.ldy + (size_t)2 * HD * h + HD + c * kAttnSlice + tid] : 0.0f;
    __syncthreads();

    // 1. scores of this CTA's positions
    const float scale = inv_sqrt_ref((float)HD);
    const float *K = L.kc + (size_t)g * d.max_ctx * HD;
    const int p0 = (int)c * per, p1 = min(np, p0 + per);
    const int k4 = tid & 3;
    const float4 *q4 = reinterpret_cast<const float4 *>(q);
    for (int base = p0; base < p1; base += HD / 4) {
        const int pp = base + (tid >> 2);
        const bool act = pp < p1;
        const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)(act ? pp : p0) * HD) + k4;
        float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
#pragma unroll
        for (int i = 0; i < HD / 16; i++) {
            const float4 kv = __ldg(kr + 4 * i), qv = q4[4 * i + k4];
            c0 = madd(c0, qv.x, kv.x);
            c1 = madd(c1, qv.y, kv.y);
            c2 = madd(c2, qv.z, kv.z);
            c3 = madd(c3, qv.w, kv.w);
        }
        const float hh = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
        const float pr = __fadd_rn(hh, __shfl_xor_sync(0xffffffffu, hh, 1));
        const float sc = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 2));
        if (act && k4 == 0) part[pp - p0] = __fmul_rn(__fadd_rn(sc, 0.0f), scale);
    }
    cluster_arrive();
    cluster_wait();

    // 2. gather every score, then the softmax (as k_attn2)
    for (int p = tid; p < np; p += HD) {
        const int owner = p / per;
        att[p] = ld_dsmem(part + (p - owner * per), (uint32_t)owner);
    }
    cluster_arrive();   // this CTA is done reading its peers; waited on before exit
    __syncthreads();
    float m = -INFINITY;
    for (int p = tid; p < np; p += HD) m = fmaxf(m, att[p]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid < 32) {
        float mm = tid < nw ? red[tid] : -INFINITY;
        for (int o = 16; o; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        if (tid == 0) s_mx = mm;
    }
    __syncthreads();
    const float mx = s_mx;
    for (int p = tid; p < np; p += HD) att[p] = pf_expf(__fadd_rn(att[p], -mx));
    __syncthreads();
    if (tid < 32) {
        const float sum = sum4_ref(att, np);
        if (tid == 0) s_inv = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int p = tid; p < np; p += HD) att[p] = __fmul_rn(att[p], inv);
    cp_async_wait<0>();   // the first kAttnRing - 1 chunks, every thread's copies
    __syncthreads();

    // 3. ordered PV chain for this CTA's 32 columns (warp 0, chunk by chunk through the ring:
    // its lanes wait for their copies of chunk ch, then refill the slot chunk ch - 1 used), gate, A8
    float o = 0.0f;
    const float *vp = vs + lane;
    for (int ch = 0; ch < nch && warp == 0; ch++) {
        if (ch > 0) {   // chunk ch (>= kAttnRing - 1: this warp's copies) landed, ch - 1 consumed
            cp_async_wait<kAttnRing - 2>();
            __syncwarp();
        }
        issue_chunk(ch + kAttnRing - 1);
        {
            const float *cv = vp + (size_t)(ch % kAttnRing) * kAttnChunk * kAttnSlice;
            const int p0c = ch * kAttnChunk, rows = min(kAttnChunk, np - p0c);
            int i = 0;
            for (; i + 8 <= rows; i += 8) {
                float v[8], a[8];
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    v[r] = cv[(size_t)(i + r) * kAttnSlice];
                    a[r] = att[p0c + i + r];
                }
#pragma unroll
                for (int r = 0; r < 8; r++) o = madd(o, a[r], v[r]);
            }
            for (; i < rows; i++) o = madd(o, att[p0c + i], cv[(size_t)i * kAttnSlice]);
        }
    }
    cp_async_wait<0>();   // the empty trailing groups
    if (warp == 0) {
        o = __fmul_rn(o, pf_sigmoid(gate));
        const int col = h * HD + (int)c * kAttnSlice, nbo = out.cols >> 5;
        quant_block_warp(o, lane, out.q + (size_t)row * out.cols + col, out.d + (size_t)row * nbo + (col >> 5),
                         out.fs + (size_t)row * nbo + (col >> 5));
    }
    cluster_wait();
}

// Grouped form of k_attn3 for multi-sequence passes: one cluster of kAttnCL CTAs per
// (sequence, KV head g, chunk of kAttnQ / G rows), G = nq / nkv query heads per KV head, so the
// cluster's up to kAttnQ queries (rows x heads of the group) share every K and V row it reads.
// Per query the arithmetic is k_attn3's (scores with pf_dot's 16-lane order over this CTA's
// positions, the full softmax in every CTA from the gathered scores: fmaxf max, pf_expf,
// sum4_ref, one division, scaling; the P.V chain of this CTA's 32 columns in position order;
// sigmoid gate; A8), so every output bit equals it. Positions are split over the CTAs by the
// group's longest causal span; PV runs on all 8 warps, two queries per warp.
constexpr int kAttnQ = 16;     // queries per cluster
constexpr int kAttn4Ring = 8;  // V chunks in flight

size_t attn4_smem(int max_ctx) {
    const size_t per = ((size_t)max_ctx + kAttnCL - 1) / kAttnCL;
    const size_t npad = ((size_t)max_ctx + 3) & ~(size_t)3;
    return sizeof(float) * ((size_t)kAttnQ * kAttnHd + (size_t)kAttnQ * ((per + 3) & ~(size_t)3) +
                            (size_t)kAttnQ * npad + (size_t)kAttn4Ring * kAttnChunk * kAttnSlice);
}

__global__ void __cluster_dims__(kAttnCL, 1, 1) __launch_bounds__(kAttnHd)
    k_attn4(AttnLayer L, AttnDims d, const float *y, const float *qbuf, const Step *st, Act out) {
    pdl_wait();
    pdl_trigger();
    constexpr int HD = kAttnHd;
    const int G = d.nq / d.nkv, QR = kAttnQ / G;            // heads per group, rows per cluster
    const int nch = (d.rps + QR - 1) / QR;
    const int g = blockIdx.y / nch, rc = blockIdx.y % nch, seq = blockIdx.z, tid = threadIdx.x;
    st += seq;
    const int n = st->n, t0 = rc * QR;
    if (t0 >= n) return;                                     // uniform over the cluster
    const int nt = min(QR, n - t0), Q = nt * G;              // live queries: q = ti * G + hh
    const int pos0 = st->pos0 + t0;
    if (pos0 >= d.max_ctx) return;
    const int np_max = min(pos0 + nt, d.max_ctx);            // longest causal span of the group
    L.kc += seq * d.ss_kv;
    L.vc += seq * d.ss_kv;
    const uint32_t c = cluster_rank();
    const int lane = tid & 31, warp = tid >> 5;
    const int per_max = (d.max_ctx + kAttnCL - 1) / kAttnCL, perp = (per_max + 3) & ~3;
    const int npad = (d.max_ctx + 3) & ~3;
    extern __shared__ __align__(16) float asm4[];
    float *qv = asm4;                                        // [kAttnQ][HD]
    float *part = qv + kAttnQ * HD;                          // [kAttnQ][perp]: this CTA's scores
    float *att = part + kAttnQ * perp;                       // [kAttnQ][npad]
    float *vs = att + (size_t)kAttnQ * npad;                 // V ring [kAttn4Ring][kAttnChunk][32]
    const int per = (np_max + kAttnCL - 1) / kAttnCL;        // positions per CTA (<= per_max)

    const float *V = L.vc + (size_t)g * d.max_ctx * HD + c * kAttnSlice;
    const int nvch = (np_max + kAttnChunk - 1) / kAttnChunk;
    auto issue_chunk = [&](int ch) {
        const int r = ch * kAttnChunk + (tid >> 3), k = tid & 7;
        if (ch < nvch && r < np_max)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                         ::"r"(smem_u32(vs + ((size_t)(ch % kAttn4Ring) * kAttnChunk + (tid >> 3)) * kAttnSlice + 4 * k)),
                         "l"(V + (size_t)r * HD + 4 * k) : "memory");
        cp_async_commit();
    };
    for (int ch = 0; ch < kAttn4Ring - 1; ch++) issue_chunk(ch);
    for (int i = tid; i < Q * HD; i += HD) {
        const int q = i / HD, ti = q / G, h = g * G + q % G;
        qv[i] = qbuf[((size_t)(st->row0 + t0 + ti) * d.nq + h) * HD + (i % HD)];
    }
    __syncthreads();

    // 1. scores of this CTA's positions for every query of the group: the K row fragment is
    // loaded once and used for all of them
    const float scale = inv_sqrt_ref((float)HD);
    const float *K = L.kc + (size_t)g * d.max_ctx * HD;
    const int p0 = (int)c * per, p1 = min(np_max, p0 + per);
    const int k4 = tid & 3;
    for (int base = p0; base < p1; base += HD / 4) {
        const int pp = base + (tid >> 2);
        const bool act = pp < p1;
        const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)(act ? pp : p0) * HD) + k4;
        float4 kf[HD / 16];
#pragma unroll
        for (int i = 0; i < HD / 16; i++) kf[i] = __ldg(kr + 4 * i);
        for (int q = 0; q < Q; q++) {
            const float4 *q4 = reinterpret_cast<const float4 *>(qv + (size_t)q * HD);
            float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
#pragma unroll
            for (int i = 0; i < HD / 16; i++) {
                const float4 qq = q4[4 * i + k4];
                c0 = madd(c0, qq.x, kf[i].x);
                c1 = madd(c1, qq.y, kf[i].y);
                c2 = madd(c2, qq.z, kf[i].z);
                c3 = madd(c3, qq.w, kf[i].w);
            }
            const float hh = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
            const float pr = __fadd_rn(hh, __shfl_xor_sync(0xffffffffu, hh, 1));
            const float sc = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 2));
            if (act && k4 == 0) part[(size_t)q * perp + (pp - p0)] = __fmul_rn(__fadd_rn(sc, 0.0f), scale);
        }
    }
    cluster_arrive();
    cluster_wait();

    // 2. every query's scores from their owners, then its softmax (one warp per query)
    for (int i = tid; i < Q * np_max; i += HD) {
        const int q = i / np_max, p = i % np_max;
        const int np = pos0 + q / G + 1;
        if (p < np) {
            const int owner = p / per;
            att[(size_t)q * npad + p] = ld_dsmem(part + (size_t)q * perp + (p - owner * per), (uint32_t)owner);
        }
    }
    cluster_arrive();   // this CTA is done reading its peers; waited on before exit
    __syncthreads();
    for (int q = warp; q < Q; q += HD / 32) {
        float *a = att + (size_t)q * npad;
        const int np = pos0 + q / G + 1;
        float m = -INFINITY;
        for (int p = lane; p < np; p += 32) m = fmaxf(m, a[p]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        for (int p = lane; p < np; p += 32) a[p] = pf_expf(__fadd_rn(a[p], -m));
        __syncwarp();
        const float sum = sum4_ref(a, np);
        const float inv = __fdiv_rn(1.0f, sum);
        for (int p = lane; p < np; p += 32) a[p] = __fmul_rn(a[p], inv);
    }

    // 3. ordered PV chains of this CTA's 32 columns, two queries per warp, chunk by chunk
    // through the V ring; gate and A8
    const int qa = warp, qb = warp + HD / 32;
    const int npa = qa < Q ? pos0 + qa / G + 1 : 0, npb = qb < Q ? pos0 + qb / G + 1 : 0;
    const float *aa = att + (size_t)(qa < Q ? qa : 0) * npad, *ab = att + (size_t)(qb < Q ? qb : 0) * npad;
    float oa = 0.0f, ob = 0.0f;
    for (int ch = 0; ch < nvch; ch++) {
        cp_async_wait<kAttn4Ring - 2>();
        __syncthreads();
        issue_chunk(ch + kAttn4Ring - 1);
        const float *cv = vs + (size_t)(ch % kAttn4Ring) * kAttnChunk * kAttnSlice + lane;
        const int pc = ch * kAttnChunk;
        const int ra = min(kAttnChunk, npa - pc), rb = min(kAttnChunk, npb - pc);
        for (int i = 0; i < ra; i++) oa = madd(oa, aa[pc + i], cv[(size_t)i * kAttnSlice]);
        for (int i = 0; i < rb; i++) ob = madd(ob, ab[pc + i], cv[(size_t)i * kAttnSlice]);
    }
    cp_async_wait<0>();
    const int nbo = out.cols >> 5;
    for (int k = 0; k < 2; k++) {
        const int q = k ? qb : qa;
        if (q >= Q) continue;
        const int h = g * G + q % G, row = st->row0 + t0 + q / G;
        const float gate = y[(size_t)row * d.ldy + (size_t)2 * HD * h + HD + c * kAttnSlice + lane];
        const float o = __fmul_rn(k ? ob : oa, pf_sigmoid(gate));
        const int col = h * HD + (int)c * kAttnSlice;
        quant_block_warp(o, lane, out.q + (size_t)row * out.cols + col, out.d + (size_t)row * nbo + (col >> 5),
                         out.fs + (size_t)row * nbo + (col >> 5));
    }
    cluster_wait();
}

// Throughput form of the grouped attention for multi-sequence passes: one CTA (no cluster) per
// (sequence, KV head g, chunk of kAttnQ / G rows), sized for many concurrent groups rather than
// for the latency of one. Per query the arithmetic is k_attn3's: scores with pf_dot's 16-lane
// order (4 threads per score; the K row fragment is loaded once into registers and used for all
// the group's queries), the softmax (fmaxf max, pf_expf, sum4_ref's 4-lane sum order, one
// division, scaling), P.V in position order from zero, sigmoid gate, A8. The probabilities are
// kept position-major (att[p][q]), so the P.V loop reads a position's 16 values with four
// 16-byte loads; thread j owns output column j of all the group's queries (16 independent
// chains), with V read 8 positions ahead (32 for QS <= 8). QS = G (one row per CTA) is the prefill
// form: a chunk's rows over a long context get many CTAs and a probability table that fits
// shared memory at 4096 positions.
template <int QS = kAttnQ>
size_t attn5_smem(int max_ctx) {
    return sizeof(float) * ((size_t)QS * kAttnHd + (((size_t)max_ctx + 3) & ~(size_t)3) * QS);
}

// sum4_ref over a[i * stride], i < n (the same 4-lane order and final combination)
__device__ float sum4_strided(const float *a, int stride, int n) {
    const int lane = threadIdx.x & 31;
    float c = 0.0f;
    const int n4 = n & ~3;
    if (lane < 4) {
        for (int i = lane; i < n4; i += 4) c = __fadd_rn(c, a[(size_t)i * stride]);
    } else if (lane == 4) {
        for (int i = n4; i < n; i++) c = __fadd_rn(c, a[(size_t)i * stride]);
    }
    const float c1 = __shfl_sync(0xffffffffu, c, 1), c2 = __shfl_sync(0xffffffffu, c, 2);
    const float c3 = __shfl_sync(0xffffffffu, c, 3), t = __shfl_sync(0xffffffffu, c, 4);
    const float c0 = __shfl_sync(0xffffffffu, c, 0);
    return __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), t);
}

template <int QS = kAttnQ>
__global__ void __launch_bounds__(kAttnHd)
    k_attn5(AttnLayer L, AttnDims d, const float *y, const float *qbuf, const Step *st, Act out) {
    pdl_wait();
    pdl_trigger();
    constexpr int HD = kAttnHd;   // att row stride: QS queries
    static_assert(QS % 4 == 0, "att rows are read as float4");
    const int G = d.nq / d.nkv, QR = QS / G;
    const int nch = (d.rps + QR - 1) / QR;
    const int g = blockIdx.x / nch, rc = blockIdx.x % nch, seq = blockIdx.y, tid = threadIdx.x;
    st += seq;
    const int n = st->n, t0 = rc * QR;
    if (t0 >= n) return;
    const int nt = min(QR, n - t0), Q = nt * G;   // live queries: q = ti * G + hh
    const int pos0 = st->pos0 + t0;
    if (pos0 >= d.max_ctx) return;
    const int np_max = min(pos0 + nt, d.max_ctx), np_min = pos0 + 1;
    L.kc += seq * d.ss_kv;
    L.vc += seq * d.ss_kv;
    const int lane = tid & 31, warp = tid >> 5;
    extern __shared__ __align__(16) float asm5[];
    float *qv = asm5;               // [QS][HD]
    float *att = qv + QS * HD;      // [np][QS]
    for (int i = tid; i < QS * HD; i += HD) {
        const int q = i / HD;
        float v = 0.0f;
        if (q < Q) {
            const int ti = q / G, h = g * G + q % G;
            v = qbuf[((size_t)(st->row0 + t0 + ti) * d.nq + h) * HD + (i % HD)];
        }
        qv[i] = v;
    }
    __syncthreads();

    // 1. scores: 64 positions per pass, 4 threads per position, all queries per K fragment. With
    // few queries per fragment (QS <= 8) the next pass's fragment is requested before this pass's
    // products, so the L2 latency is not paid per pass; with 16 the registers go to occupancy.
    const float scale = inv_sqrt_ref((float)HD);
    const float *K = L.kc + (size_t)g * d.max_ctx * HD;
    const int k4 = tid & 3;
    constexpr bool PIPE = QS <= 8;
    float4 kn[PIPE ? HD / 16 : 1];
    if constexpr (PIPE) {
        const int pp = tid >> 2;
        const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)(pp < np_max ? pp : 0) * HD) + k4;
#pragma unroll
        for (int i = 0; i < HD / 16; i++) kn[i] = __ldg(kr + 4 * i);
    }
    for (int base = 0; base < np_max; base += HD / 4) {
        const int pp = base + (tid >> 2);
        const bool act = pp < np_max;
        float4 kf[HD / 16];
        if constexpr (PIPE) {
#pragma unroll
            for (int i = 0; i < HD / 16; i++) kf[i] = kn[i];
            if (base + HD / 4 < np_max) {
                const int pn = pp + HD / 4;
                const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)(pn < np_max ? pn : 0) * HD) + k4;
#pragma unroll
                for (int i = 0; i < HD / 16; i++) kn[i] = __ldg(kr + 4 * i);
            }
        } else {
            const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)(act ? pp : 0) * HD) + k4;
#pragma unroll
            for (int i = 0; i < HD / 16; i++) kf[i] = __ldg(kr + 4 * i);
        }
        for (int q = 0; q < Q; q++) {
            const float4 *q4 = reinterpret_cast<const float4 *>(qv + (size_t)q * HD);
            float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
#pragma unroll
            for (int i = 0; i < HD / 16; i++) {
                const float4 qq = q4[4 * i + k4];
                c0 = madd(c0, qq.x, kf[i].x);
                c1 = madd(c1, qq.y, kf[i].y);
                c2 = madd(c2, qq.z, kf[i].z);
                c3 = madd(c3, qq.w, kf[i].w);
            }
            const float hh = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
            const float pr = __fadd_rn(hh, __shfl_xor_sync(0xffffffffu, hh, 1));
            const float sc = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 2));
            if (act && k4 == 0) att[(size_t)pp * QS + q] = __fmul_rn(__fadd_rn(sc, 0.0f), scale);
        }
    }
    __syncthreads();

    // 2. softmax of each query over its causal span (one warp per query)
    for (int q = warp; q < Q; q += HD / 32) {
        const int np = pos0 + q / G + 1;
        float m = -INFINITY;
        for (int p = lane; p < np; p += 32) m = fmaxf(m, att[(size_t)p * QS + q]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        for (int p = lane; p < np; p += 32) att[(size_t)p * QS + q] = pf_expf(__fadd_rn(att[(size_t)p * QS + q], -m));
        __syncwarp();
        const float sum = sum4_strided(att + q, QS, np);
        const float inv = __fdiv_rn(1.0f, sum);
        for (int p = lane; p < np; p += 32) att[(size_t)p * QS + q] = __fmul_rn(att[(size_t)p * QS + q], inv);
    }
    __syncthreads();

    // 3. P.V: column tid of every query, positions in order; every query is live over
    // [0, np_min), the group's later rows over their longer spans after that
    const float *V = L.vc + (size_t)g * d.max_ctx * HD + tid;
    float acc[QS];
#pragma unroll
    for (int q = 0; q < QS; q++) acc[q] = 0.0f;
    constexpr int PF = QS <= 8 ? 32 : 8;   // V rows in flight: a few queries' chains are short
    float vn[PF];
#pragma unroll
    for (int i = 0; i < PF; i++) vn[i] = i < np_min ? __ldg(V + (size_t)i * HD) : 0.0f;
    int p = 0;
    for (; p + PF <= np_min; p += PF) {
        float vc[PF];
#pragma unroll
        for (int i = 0; i < PF; i++) {
            vc[i] = vn[i];
            const int pn = p + PF + i;
            vn[i] = pn < np_min ? __ldg(V + (size_t)pn * HD) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < PF; i++) {
            const float4 *a4 = reinterpret_cast<const float4 *>(att + (size_t)(p + i) * QS);
#pragma unroll
            for (int j = 0; j < QS / 4; j++) {
                const float4 a = a4[j];
                acc[4 * j] = madd(acc[4 * j], a.x, vc[i]);
                acc[4 * j + 1] = madd(acc[4 * j + 1], a.y, vc[i]);
                acc[4 * j + 2] = madd(acc[4 * j + 2], a.z, vc[i]);
                acc[4 * j + 3] = madd(acc[4 * j + 3], a.w, vc[i]);
            }
        }
    }
    for (; p < np_max; p++) {
        const float v = __ldg(V + (size_t)p * HD);
        const float4 *a4 = reinterpret_cast<const float4 *>(att + (size_t)p * QS);
#pragma unroll
        for (int j = 0; j < QS / 4; j++) {
            const float4 a = a4[j];
            const float aq[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int q = 4 * j + r;
                if (q < Q && p < pos0 + q / G + 1) acc[q] = madd(acc[q], aq[r], v);
            }
        }
    }

    // 4. gate and A8: warp w's 32 columns are one block of each query's output row
    const int nbo = out.cols >> 5;
#pragma unroll
    for (int q = 0; q < QS; q++) {
        if (q >= Q) break;
        const int h = g * G + q % G, row = st->row0 + t0 + q / G;
        const float gate = y[(size_t)row * d.ldy + (size_t)2 * HD * h + HD + tid];
        const float o = __fmul_rn(acc[q], pf_sigmoid(gate));
        const int col = h * HD + warp * 32;
        quant_block_warp(o, lane, out.q + (size_t)row * out.cols + col, out.d + (size_t)row * nbo + (col >> 5),
                         out.fs + (size_t)row * nbo + (col >> 5));
    }
}

// Gated DeltaNet layer, latency-oriented form of k_deltanet with identical per-element
// arithmetic (same citations). Differences are scheduling only:
//  - one cp.async batch brings this key head's q / k / v / z / b / a rows of every token into
//    shared memory while the 64 KB state column loads into registers;
//  - the conv runs with its taps in registers (conv_k == KC);
//  - the deferred-commit replay is folded into token 0's first sweep (kern_lin.c replay_first,
//    :42-62: per element the same operations in the same order), and token t's second sweep
//    (S += k delta; o += S q) runs in the same loop as token t+1's first sweep (S *= decay;
//    kv += S k), two independent add chains per iteration.
// rep == 1 only (one value head per key head, every Qwen3.5 size); KC taps.

// One conv channel of k_deltanet2 held in registers (every array index a constant): the state
// rows, the taps, and the conv-log rows a pending commit shifts in (pf_lin_commit's conv part,
// kern_lin.c: new state row r = old row r + e1 while that exists, else logged input row
// r + e1 - S + 1, e1 = pend_conv - 1).
// A global load issued where it is written: volatile asm keeps its place among the other
// volatile asm of the kernel (the cp.async copies), so the compiler cannot sink it to the first
// use to save registers; the value is waited for only where it is used.
__device__ __forceinline__ float ld_early(const float *p) {
    float v;
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

template <int KC>
struct ConvCh {
    static constexpr int S = KC - 1;
    float st[S > 0 ? S : 1], w[KC], xr[S > 0 ? S : 1];
    int c;
};
template <int KC>
__device__ __forceinline__ void conv_load(ConvCh<KC> &ch, const LinLayer &L, int C, int c) {
    constexpr int S = KC - 1;
    ch.c = c;
#pragma unroll
    for (int r = 0; r < S; r++) ch.st[r] = ld_early(L.conv_state + (size_t)r * C + c);
#pragma unroll
    for (int r = 0; r < KC; r++) ch.w[r] = ld_early(L.conv_w + (size_t)c * KC + r);
}
template <int KC>
__device__ __forceinline__ void conv_load_log(ConvCh<KC> &ch, const LinLayer &L, int C, int pend_conv) {
    constexpr int S = KC - 1;
    const int c = ch.c;
    const int e1 = pend_conv - 1;
#pragma unroll
    for (int r = 0; r < S; r++) {
        const int src = r + e1;
        ch.xr[r] = (pend_conv > 1 && src >= S) ? ld_early(L.xin + (size_t)(src - S + 1) * C + c) : 0.0f;
    }
}
template <int KC>
__device__ __forceinline__ void conv_commit(ConvCh<KC> &ch, int pend_conv) {
    constexpr int S = KC - 1;
    if (pend_conv > 1) {
        const int e1 = pend_conv - 1;
        float ns[S > 0 ? S : 1];
#pragma unroll
        for (int r = 0; r < S; r++) {
            const int src = r + e1;
            float v = ch.xr[r];
#pragma unroll
            for (int q2 = 0; q2 < S; q2++)
                if (src == q2) v = ch.st[q2];
            ns[r] = v;
        }
#pragma unroll
        for (int r = 0; r < S; r++) ch.st[r] = ns[r];
    }
}
// conv tap sum of token t (state rows, then the token's own input), state shift, SiLU
template <int KC>
__device__ __forceinline__ float conv_step(ConvCh<KC> &ch, float xc) {
    constexpr int S = KC - 1;
    float acc = __fmul_rn(ch.w[0], S > 0 ? ch.st[0] : xc);
#pragma unroll
    for (int r = 1; r < KC; r++) acc = madd(acc, ch.w[r], r < S ? ch.st[r < S ? r : 0] : xc);
#pragma unroll
    for (int r = 0; r + 1 < S; r++) ch.st[r] = ch.st[r + 1];
    if (S > 0) ch.st[S - 1] = xc;
    return pf_silu(acc);
}
template <int KC>
__device__ __forceinline__ void conv_store(const ConvCh<KC> &ch, const LinLayer &L, int C, const float *live,
                                           int logged) {
    constexpr int S = KC - 1;
#pragma unroll
    for (int r = 0; r < S; r++) L.conv_state[(size_t)r * C + ch.c] = logged ? live[r] : ch.st[r];
}


// 8 rows i0..i0+7 of a state column (stride kDV) / 8 consecutive floats (16-byte aligned)
__device__ __forceinline__ void ld8col(float (&v)[8], const float *col, int i0) {
#pragma unroll
    for (int r = 0; r < 8; r++) v[r] = col[(size_t)(i0 + r) * kDV];
}
__device__ __forceinline__ void st8col(float *col, int i0, const float (&v)[8]) {
#pragma unroll
    for (int r = 0; r < 8; r++) col[(size_t)(i0 + r) * kDV] = v[r];
}
__device__ __forceinline__ void ld8(float (&v)[8], const float *p) {
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// NR: the most rows a pass may have (the shared-memory row buffers; a 4-row variant serves
// multi-sequence verify passes, where a smaller footprint fits three CTAs on an SM). RP: the
// most deferred updates a pass may replay (the last commit's rows after its first: up to
// PINFER_SPEC_MAX_K on a context, the batch's draft depth on a batch); the replay is unrolled
// over RP, so each launch takes the smallest variant that holds its bound.
template <int KC, int NR = kMaxRows, int RP = NR - 1>
__global__ void __launch_bounds__(128, 1) k_deltanet2(LinLayer L, LinDims d, const float *y, Step *st,
                                                      Act out) {
    constexpr int S = KC - 1;
    const int h = blockIdx.x, j = threadIdx.x;
    const int C = d.C;
    // blockIdx.y: the sequence of a multi-sequence batch (its states, Step block and rows)
    const int seq = blockIdx.y;
    st += seq;
    L.conv_state += seq * d.ss_conv;
    L.rec += seq * d.ss_rec;
    L.xin += seq * d.ss_xin;
    L.upd += seq * d.ss_upd;
    // conv taps and state rows of this thread's three channels (q, k, v column j of this
    // head): independent of the step and the first thing the kernel needs, so requested first
    ConvCh<KC> cq, ck, cv;
    conv_load(cq, L, C, h * kDK + j);
    conv_load(ck, L, C, d.kd + h * kDK + j);
    conv_load(cv, L, C, 2 * d.kd + h * kDV + j);
    // ---- prefetch by TMA bulk copies: the 64 KB state on sbar[1] (before pdl_wait: only this
    // kernel writes it), after pdl_wait this head's q / k / v / z rows of every token on
    // sbar[0]. Bulk copies do not queue in the SM's load / store path, so the loads and stores
    // below do not wait behind the state. Rows are 512 B at 16-byte aligned offsets
    // (launch_deltanet checks ldy).
    __shared__ __align__(8) uint64_t sbar[2];
    extern __shared__ __align__(16) float Ssm[];   // [kDK][kDV]: this head's state, row-major
    if (j == 0) {
        mbar_init(&sbar[0], 1);
        mbar_init(&sbar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const float *rec_h = L.rec + (size_t)h * kDK * kDV;
    if (j == 0) {
        mbar_arrive_expect(&sbar[1], kDK * kDV * 4);
        for (int q4 = 0; q4 < 4; q4++)
            bulk_g2s(Ssm + q4 * (kDK * kDV / 4), rec_h + q4 * (kDK * kDV / 4), kDK * kDV, &sbar[1]);
    }
    pdl_wait();
    pdl_trigger();
    const int n = st->n;
    if (n <= 0 || n > NR || st->pend_keep > RP) {   // nothing to do (or more rows / replayed
        // updates than this variant holds: reported); the state copy lands before smem goes
        if ((n > NR || st->pend_keep > RP) && j == 0) st->status = -92;
        mbar_wait(&sbar[1], 0);
        return;
    }
    const int row0 = st->row0;
    const int logged = st->logged, pend_keep = st->pend_keep, pend_conv = st->pend_conv;
    const int wr = st->wr;
    conv_load_log(cq, L, C, pend_conv);
    conv_load_log(ck, L, C, pend_conv);
    conv_load_log(cv, L, C, pend_conv);
    __shared__ __align__(16) float sq[NR][kDK], sk[NR][kDK], sv[NR][kDV];
    __shared__ __align__(16) float sz[NR][kDV];
    // token t's output row reuses its v row: thread j reads v[t][j] at the start of token t and
    // writes o[t][j] at its end, and no other thread reads column j of either
    float (*so)[kDV] = sv;
    __shared__ float sbeta[NR], sdec[NR], srn[NR];
    __shared__ __align__(16) float skp[RP][kDK];
    __shared__ float spd[RP];
    const size_t logw = (size_t)kDK + kDV + 1;

    if (j == 0) {
        mbar_arrive_expect(&sbar[0], (uint32_t)n * 4u * kDK * 4u);
        for (int t = 0; t < n; t++) {
            const float *yr = y + (size_t)(row0 + t) * d.ldy;
            bulk_g2s(sq[t], yr + h * kDK, kDK * 4, &sbar[0]);
            bulk_g2s(sk[t], yr + d.kd + h * kDK, kDK * 4, &sbar[0]);
            bulk_g2s(sv[t], yr + 2 * d.kd + h * kDV, kDV * 4, &sbar[0]);
            bulk_g2s(sz[t], yr + C + h * kDV, kDV * 4, &sbar[0]);
        }
    }
    const int keep = pend_keep;   // <= RP (checked above)
    float dl[RP];
#pragma unroll
    for (int tp = 0; tp < RP; tp++) {   // deferred commit: rows 1..keep of half wr^1
        dl[tp] = 0.0f;
        if (tp < keep) {
            const float *u = L.upd + (((size_t)(wr ^ 1) * d.cap + tp + 1) * d.nv + h) * logw;
            skp[tp][j] = u[j];
            dl[tp] = u[kDK + j];
            if (j == 0) spd[tp] = u[kDK + kDV];
        }
    }
    float *rec = L.rec + (size_t)h * kDK * kDV + j;
    float *Sj = Ssm + j;   // column j: Sj[i * kDV]
    // ---- gates of token t on thread kDV - NR + t (warp 3), while the state streams in
    if (j >= kDV - NR && j - (kDV - NR) < n) {
        const int t = j - (kDV - NR);
        const float *yr = y + (size_t)(row0 + t) * d.ldy;
        const float b = yr[C + d.vd + h], a = yr[C + d.vd + d.nv + h];
        sbeta[t] = __fdiv_rn(1.0f, __fadd_rn(1.0f, glibc_expf(-b)));
        const float xs = __fadd_rn(a, L.dt_bias[h]);
        const float sp = xs > 20.0f ? xs : glibc_log1pf(glibc_expf(xs));
        sdec[t] = glibc_expf(__fmul_rn(L.A[h], sp));
    }
    if (!mbar_wait(&sbar[0], 0)) {   // the rows: timed out, reported, no hang; a second
        if (j == 0) st->status = -90;   // bounded wait lets the copies in flight land
        mbar_wait(&sbar[0], 0);
    }
    __syncthreads();
    // ---- pending conv commit, then conv + SiLU for the three channels
    // (the three channels advance together: three independent chains per token)
    conv_commit(cq, pend_conv);
    conv_commit(ck, pend_conv);
    conv_commit(cv, pend_conv);
    {
        float lq[S > 0 ? S : 1], lk[S > 0 ? S : 1], lv[S > 0 ? S : 1];
#pragma unroll
        for (int r = 0; r < S; r++) lq[r] = lk[r] = lv[r] = 0.0f;
        for (int t = 0; t < n; t++) {
            const float xq = sq[t][j], xk = sk[t][j], xv = sv[t][j];
            const float oq = conv_step(cq, xq), ok = conv_step(ck, xk), ov = conv_step(cv, xv);
            sq[t][j] = oq;
            sk[t][j] = ok;
            sv[t][j] = ov;
            if (logged) {
                if (t == 0) {
#pragma unroll
                    for (int r = 0; r < S; r++) {
                        lq[r] = cq.st[r];
                        lk[r] = ck.st[r];
                        lv[r] = cv.st[r];
                    }
                } else {
                    L.xin[(size_t)t * C + cq.c] = xq;
                    L.xin[(size_t)t * C + ck.c] = xk;
                    L.xin[(size_t)t * C + cv.c] = xv;
                }
            }
        }
        conv_store(cq, L, C, lq, logged);
        conv_store(ck, L, C, lk, logged);
        conv_store(cv, L, C, lv, logged);
    }
    __syncthreads();
    // ---- L2 norm of q and k: 4 lanes per (token, vector)
    {
        const int lane = j & 31, warp = j >> 5;
        const float qscale = inv_sqrt_ref((float)kDK);
        for (int u0 = warp * 8; u0 < 2 * n; u0 += 4 * 8) {
            const int u = u0 + (lane >> 2), l = lane & 3;
            const bool act = u < 2 * n;
            float *vec = act ? ((u & 1) ? sk[u >> 1] : sq[u >> 1]) : sq[0];
            float c = 0.0f;
            if (act) {
#pragma unroll 32
                for (int i = l; i < kDK; i += 4) c = madd(c, vec[i], vec[i]);
            }
            const int base = lane & ~3;
            const float c0 = __shfl_sync(0xffffffffu, c, base), c1 = __shfl_sync(0xffffffffu, c, base + 1);
            const float c2 = __shfl_sync(0xffffffffu, c, base + 2), c3 = __shfl_sync(0xffffffffu, c, base + 3);
            const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
            const float r = inv_sqrt_ref(__fadd_rn(ss, 1e-6f));
            __syncwarp();
            if (act) {
                const float sc = (u & 1) ? 1.0f : qscale;
                for (int i = l; i < kDK; i += 4) vec[i] = __fmul_rn(__fmul_rn(vec[i], r), sc);
            }
        }
    }
    if (!mbar_wait(&sbar[1], 0)) {   // the state: timed out, reported, no hang; a second
        if (j == 0) st->status = -90;   // bounded wait lets the copies in flight land
        mbar_wait(&sbar[1], 0);
    }
    __syncthreads();

    // ---- recurrence: replay + token 0 first sweep, then fused sweeps (column j in smem).
    // The column moves through registers 8 rows at a time, the next 8 rows loaded before this
    // chunk is stored back (the compiler cannot prove the state and the q / k rows disjoint, so
    // it would not hoist those loads itself); per element the operations and their order are
    // unchanged, and the dot-product chains still run over i = 0..kDK-1 in order.
    float kv = 0.0f;
    {
        const float dec = sdec[0];
        const float *k0 = sk[0];
        float sc[8];
        ld8col(sc, Sj, 0);
        for (int i0 = 0; i0 < kDK; i0 += 8) {
            float sn[8], k8[8];
            ld8col(sn, Sj, i0 + 8 < kDK ? i0 + 8 : i0);
            ld8(k8, k0 + i0);
#pragma unroll
            for (int tp = 0; tp < RP; tp++) {
                if (tp < keep) {
                    float kp[8];
                    ld8(kp, skp[tp] + i0);
                    const float pd = spd[tp];
#pragma unroll
                    for (int r = 0; r < 8; r++) sc[r] = __fadd_rn(__fmul_rn(sc[r], pd), __fmul_rn(kp[r], dl[tp]));
                }
            }
#pragma unroll
            for (int r = 0; r < 8; r++) {
                sc[r] = __fmul_rn(sc[r], dec);
                kv = madd(kv, sc[r], k8[r]);
            }
            st8col(Sj, i0, sc);
#pragma unroll
            for (int r = 0; r < 8; r++) sc[r] = sn[r];
        }
    }
    for (int t = 0; t < n; t++) {
        const float delta = __fmul_rn(__fadd_rn(sv[t][j], -kv), sbeta[t]);
        const float *kt = sk[t], *qt = sq[t];
        float o = 0.0f, kvn = 0.0f;
        const bool next = t + 1 < n;
        const float decn = next ? sdec[t + 1] : 0.0f;
        const float *kn = sk[next ? t + 1 : t];
        const bool store_live = logged && t == 0;
        const bool store_rec = store_live || (!next && !logged);
        float sc[8];
        ld8col(sc, Sj, 0);
        for (int i0 = 0; i0 < kDK; i0 += 8) {
            float sn[8], k8[8], q8[8];
            ld8col(sn, Sj, i0 + 8 < kDK ? i0 + 8 : i0);
            ld8(k8, kt + i0);
            ld8(q8, qt + i0);
            if (next) {
                float n8[8];
                ld8(n8, kn + i0);
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    float sv_ = __fadd_rn(sc[r], __fmul_rn(k8[r], delta));
                    o = madd(o, sv_, q8[r]);
                    if (store_live) rec[(size_t)(i0 + r) * kDV] = sv_;
                    sv_ = __fmul_rn(sv_, decn);
                    kvn = madd(kvn, sv_, n8[r]);
                    sc[r] = sv_;
                }
            } else {
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    const float sv_ = __fadd_rn(sc[r], __fmul_rn(k8[r], delta));
                    o = madd(o, sv_, q8[r]);
                    sc[r] = sv_;
                    if (store_rec) rec[(size_t)(i0 + r) * kDV] = sv_;
                }
            }
            st8col(Sj, i0, sc);
#pragma unroll
            for (int r = 0; r < 8; r++) sc[r] = sn[r];
        }
        so[t][j] = o;
        if (logged && t > 0) {
            float *u = L.upd + (((size_t)wr * d.cap + t) * d.nv + h) * logw;
            u[kDK + j] = delta;
            u[j] = kt[j];
            if (j == 0) u[kDK + kDV] = sdec[t];
        }
        kv = kvn;
    }
    __syncthreads();

    // ---- gated RMSNorm and A8
    {
        const int lane = j & 31, warp = j >> 5;
        for (int u0 = warp * 8; u0 < n; u0 += 4 * 8) {
            const int u = u0 + (lane >> 2), l = lane & 3;
            const bool act = u < n;
            const float *vec = so[act ? u : 0];
            float c = 0.0f;
            if (act) {
#pragma unroll 32
                for (int i = l; i < kDV; i += 4) c = madd(c, vec[i], vec[i]);
            }
            const int base = lane & ~3;
            const float c0 = __shfl_sync(0xffffffffu, c, base), c1 = __shfl_sync(0xffffffffu, c, base + 1);
            const float c2 = __shfl_sync(0xffffffffu, c, base + 2), c3 = __shfl_sync(0xffffffffu, c, base + 3);
            const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
            if (act && l == 0) srn[u] = inv_sqrt_ref(__fadd_rn(__fdiv_rn(ss, (float)kDV), d.eps));
        }
    }
    __syncthreads();
    {
        const int lane = j & 31, warp = j >> 5, nbo = out.cols >> 5;
        const float w = L.norm_w[j];
        for (int t = 0; t < n; t++) {
            float v = __fmul_rn(__fmul_rn(so[t][j], srn[t]), w);
            v = __fmul_rn(v, pf_silu(sz[t][j]));
            const int col = h * kDV + j;
            quant_block_warp(v, lane, out.q + (size_t)(row0 + t) * out.cols + (col & ~31),
                             out.d + (size_t)(row0 + t) * nbo + (col >> 5), out.fs + (size_t)(row0 + t) * nbo + (col >> 5));
            (void)warp;
        }
    }
}


// Gated DeltaNet layer of a single context's pass, spread over a 4-CTA cluster per key head:
// the same per-element arithmetic as k_deltanet2 (same citations), scheduled for latency.
// k_deltanet2 gives each state column one thread, which then does every state update of that
// column and both of its ordered add chains: one warp per SM sub-partition, issue-bound. Here
// CTA c of the cluster owns state columns 32c..32c+31 and its warp p owns state rows
// 32p..32p+31, the state itself in registers, so every element update and product of a token
// runs on 16 warps of 4 SMs in parallel; only the adds of the ordered chains (kv and o run over
// the rows i = 0..127 in order, kern_lin.c) pass from warp to warp: warp p adds the products of
// its 32 rows to the partial sum warp p - 1 hands it through shared memory and a named barrier.
// Each CTA computes the whole q and k vectors of every token (conv, L2 norm), the gates and the
// v / z columns it owns; the gated RMSNorm runs over the head's 128 outputs, which the CTAs
// exchange through distributed shared memory; each CTA quantises its own 32-column A8 block.
// Conv states, logs and state rows are written by the CTA that owns them.
constexpr int kDnCl = 4;                    // CTAs per key head (cluster)
constexpr int kDnCols = kDV / kDnCl;        // state columns per CTA
constexpr int kDnParts = 4;                 // warps per CTA
constexpr int kDnPart = kDK / kDnParts;     // state rows per warp

__device__ __forceinline__ void bar_sync_n(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive_n(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// a float into CTA `rank`'s shared memory at the offset of `local` in this CTA's
__device__ __forceinline__ void st_dsmem(float *local, uint32_t rank, float v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// pre: the rows the pass may have; rows 0..pre-1 of this head are loaded right after pdl_wait,
// beside the Step block (the pass must start at row 0 and have at most pre rows: checked).
template <int KC, int NR, int RP>
__global__ void __cluster_dims__(kDnCl, 1, 1) __launch_bounds__(kDnParts * 32, 1)
    k_deltanet3(LinLayer L, LinDims d, const float *y, Step *st, Act out, int pre) {
    static_assert(kDnParts * 32 == kDK && kDnCols == 32 && NR <= kDnParts * 32 && RP >= 1, "shape");
    constexpr int S = KC - 1;
    constexpr int NT = (NR + kDnParts - 1) / kDnParts;   // output rows per warp (epilogue)
    const int h = blockIdx.x / kDnCl, c = (int)cluster_rank();
    const int j = threadIdx.x, w = j >> 5, lane = j & 31;
    const int col = c * kDnCols + lane;   // this thread's state column (within the head)
    const int i0 = w * kDnPart;           // its first state row
    const int C = d.C;
    // conv taps and state rows: q and k channel j (every CTA needs the whole q and k vectors),
    // v channel col (warp 0); this thread's 32 state elements. All independent of the step and
    // written only by this kernel, so requested before pdl_wait.
    ConvCh<KC> cq, ck, cv;
    conv_load(cq, L, C, h * kDK + j);
    conv_load(ck, L, C, d.kd + h * kDK + j);
    if (w == 0) conv_load(cv, L, C, 2 * d.kd + h * kDV + col);
    float *rec = L.rec + (size_t)h * kDK * kDV + col;   // rec[i * kDV]: row i of this column
    float Sr[kDnPart];
#pragma unroll
    for (int r = 0; r < kDnPart; r++) Sr[r] = ld_early(rec + (size_t)r * kDV + (size_t)i0 * kDV);
    // The pass's Step block is written only between passes (set_pass / k_accept, never by this
    // kernel's predecessor, the W_in matvec), and the conv-input log and the deferred-commit rows
    // only by this layer's own DeltaNet in an earlier pass, so all of them are read before
    // pdl_wait as well; the W_in rows are not.
    const int n = ld_early_s32(&st->n), row0 = ld_early_s32(&st->row0);
    const int logged = ld_early_s32(&st->logged), keep = ld_early_s32(&st->pend_keep);
    const int pend_conv = ld_early_s32(&st->pend_conv), wr = ld_early_s32(&st->wr);
    conv_load_log(cq, L, C, pend_conv);
    conv_load_log(ck, L, C, pend_conv);
    if (w == 0) conv_load_log(cv, L, C, pend_conv);
    const size_t logw = (size_t)kDK + kDV + 1;
    // deferred commit: rows 1..keep of half wr^1, held in registers until the first sweep
    float dl[RP], kpr[RP], pdr[RP];
#pragma unroll
    for (int tp = 0; tp < RP; tp++) {
        dl[tp] = kpr[tp] = pdr[tp] = 0.0f;
        if (tp < keep) {
            const float *u = L.upd + (((size_t)(wr ^ 1) * d.cap + tp + 1) * d.nv + h) * logw;
            kpr[tp] = ld_early(u + j);
            dl[tp] = ld_early(u + kDK + col);
            if (j == 0) pdr[tp] = ld_early(u + kDK + kDV);
        }
    }
    pdl_wait();
    pdl_trigger();
    // rows 0..pre-1: the conv inputs of this thread's channels, its z column for the output rows
    // it gates, the gate inputs (thread kDK - NR + t); requested together with the Step block
    float xq[NR], xk[NR], xv[NR], zt[NT], gb = 0.0f, ga = 0.0f;
#pragma unroll
    for (int t = 0; t < NR; t++) {
        xq[t] = xk[t] = xv[t] = 0.0f;
        if (t < pre) {
            const float *yr = y + (size_t)t * d.ldy;
            xq[t] = ld_early(yr + h * kDK + j);
            xk[t] = ld_early(yr + d.kd + h * kDK + j);
            if (w == 0) xv[t] = ld_early(yr + 2 * d.kd + h * kDV + col);
        }
    }
#pragma unroll
    for (int q = 0; q < NT; q++) {
        const int t = w + q * kDnParts;
        zt[q] = t < pre ? ld_early(y + (size_t)t * d.ldy + C + h * kDV + col) : 0.0f;
    }
    const int tg = j - (kDK - NR);   // this thread's gate row
    if (tg >= 0 && tg < pre) {
        const float *yr = y + (size_t)tg * d.ldy;
        gb = ld_early(yr + C + d.vd + h);
        ga = ld_early(yr + C + d.vd + d.nv + h);
    }
    if (n <= 0 || n > NR || n > pre || row0 != 0 || keep > RP) {   // nothing to do, or a pass
        // this variant does not hold (reported); the same for every CTA of the cluster
        if (n > 0 && j == 0 && c == 0) st->status = -92;
        return;
    }
    __shared__ __align__(16) float sq[NR][kDK], sk[NR][kDK];
    __shared__ __align__(16) float sv[NR][kDnCols];
    __shared__ __align__(16) float so[NR][kDV];   // the head's output rows
    __shared__ float sbeta[NR], sdec[NR], srn[NR];
    __shared__ __align__(16) float skp[RP][kDK];
    __shared__ float spd[RP];
    __shared__ float sdelta[kDnCols], xo[kDnParts][kDnCols], xk_[kDnParts][kDnCols];
    // ---- gates of token tg
    if (tg >= 0 && tg < n) {
        sbeta[tg] = __fdiv_rn(1.0f, __fadd_rn(1.0f, glibc_expf(-gb)));
        const float xs = __fadd_rn(ga, L.dt_bias[h]);
        const float sp = xs > 20.0f ? xs : glibc_log1pf(glibc_expf(xs));
        sdec[tg] = glibc_expf(__fmul_rn(L.A[h], sp));
    }
    // ---- pending conv commit, then conv + SiLU (q / k channel j; v channel col on warp 0)
    const bool own_qk = w == c;   // q / k channel j is this CTA's to store and log
    conv_commit(cq, pend_conv);
    conv_commit(ck, pend_conv);
    if (w == 0) conv_commit(cv, pend_conv);
    {
        float lq[S > 0 ? S : 1], lk[S > 0 ? S : 1], lv[S > 0 ? S : 1];
#pragma unroll
        for (int r = 0; r < S; r++) lq[r] = lk[r] = lv[r] = 0.0f;
#pragma unroll
        for (int t = 0; t < NR; t++) {
            if (t < n) {
                sq[t][j] = conv_step(cq, xq[t]);
                sk[t][j] = conv_step(ck, xk[t]);
                if (w == 0) sv[t][lane] = conv_step(cv, xv[t]);
                if (logged) {
                    if (t == 0) {
#pragma unroll
                        for (int r = 0; r < S; r++) {
                            lq[r] = cq.st[r];
                            lk[r] = ck.st[r];
                            lv[r] = cv.st[r];
                        }
                    } else {
                        if (own_qk) {
                            L.xin[(size_t)t * C + cq.c] = xq[t];
                            L.xin[(size_t)t * C + ck.c] = xk[t];
                        }
                        if (w == 0) L.xin[(size_t)t * C + cv.c] = xv[t];
                    }
                }
            }
        }
        if (own_qk) {
            conv_store(cq, L, C, lq, logged);
            conv_store(ck, L, C, lk, logged);
        }
        if (w == 0) conv_store(cv, L, C, lv, logged);
    }
    __syncthreads();
    // ---- L2 norm of q and k: 4 lanes per (token, vector)
    {
        const float qscale = inv_sqrt_ref((float)kDK);
        for (int u0 = w * 8; u0 < 2 * n; u0 += kDnParts * 8) {
            const int u = u0 + (lane >> 2), l = lane & 3;
            const bool act = u < 2 * n;
            float *vec = act ? ((u & 1) ? sk[u >> 1] : sq[u >> 1]) : sq[0];
            float cs = 0.0f;
            if (act) {
#pragma unroll 32
                for (int i = l; i < kDK; i += 4) cs = madd(cs, vec[i], vec[i]);
            }
            const int base = lane & ~3;
            const float c0 = __shfl_sync(0xffffffffu, cs, base), c1 = __shfl_sync(0xffffffffu, cs, base + 1);
            const float c2 = __shfl_sync(0xffffffffu, cs, base + 2), c3 = __shfl_sync(0xffffffffu, cs, base + 3);
            const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
            const float r = inv_sqrt_ref(__fadd_rn(ss, 1e-6f));
            __syncwarp();
            if (act) {
                const float sc = (u & 1) ? 1.0f : qscale;
                for (int i = l; i < kDK; i += 4) vec[i] = __fmul_rn(__fmul_rn(vec[i], r), sc);
            }
        }
    }
#pragma unroll
    for (int tp = 0; tp < RP; tp++) {
        if (tp < keep) {
            skp[tp][j] = kpr[tp];
            if (j == 0) spd[tp] = pdr[tp];
        }
    }
    __syncthreads();

    // ---- recurrence. Named barriers: 1 (all warps) publishes a token's delta; 1 + p hands
    // the partial sums of rows 0..32p-1 from warp p - 1 to warp p.
    float pk[kDnPart];
    {   // replay of the deferred commit (per element in commit order) and token 0's decay,
        // then kv over the rows in order
#pragma unroll
        for (int tp = 0; tp < RP; tp++) {
            if (tp < keep) {
                const float pd = spd[tp], dt = dl[tp];
                const float *kp = skp[tp] + i0;
#pragma unroll
                for (int r = 0; r < kDnPart; r++) Sr[r] = __fadd_rn(__fmul_rn(Sr[r], pd), __fmul_rn(kp[r], dt));
            }
        }
        const float dec = sdec[0];
        const float *k0 = sk[0] + i0;
#pragma unroll
        for (int r = 0; r < kDnPart; r++) {
            Sr[r] = __fmul_rn(Sr[r], dec);
            pk[r] = __fmul_rn(Sr[r], k0[r]);
        }
        float kv = 0.0f;
        if (w > 0) {
            bar_sync_n(1 + w, 64);
            kv = xk_[w][lane];
        }
#pragma unroll
        for (int r = 0; r < kDnPart; r++) kv = __fadd_rn(kv, pk[r]);
        if (w < kDnParts - 1) {
            xk_[w + 1][lane] = kv;
            bar_arrive_n(2 + w, 64);
        } else {
            sdelta[lane] = __fmul_rn(__fadd_rn(sv[0][lane], -kv), sbeta[0]);
        }
    }
    for (int t = 0; t < n; t++) {
        bar_sync_n(1, kDnParts * 32);   // delta of token t
        const float delta = sdelta[lane];
        const bool next = t + 1 < n;
        const float decn = next ? sdec[t + 1] : 0.0f;
        const float *kt = sk[t] + i0, *qt = sq[t] + i0, *kn = sk[next ? t + 1 : t] + i0;
        const bool store_live = logged && t == 0;
        const bool store_rec = store_live || (!next && !logged);
        float po[kDnPart];
#pragma unroll
        for (int r = 0; r < kDnPart; r++) {
            float sv_ = __fadd_rn(Sr[r], __fmul_rn(kt[r], delta));
            po[r] = __fmul_rn(sv_, qt[r]);
            if (store_rec) rec[(size_t)(i0 + r) * kDV] = sv_;
            if (next) {
                sv_ = __fmul_rn(sv_, decn);
                pk[r] = __fmul_rn(sv_, kn[r]);
            }
            Sr[r] = sv_;
        }
        float o = 0.0f, kvn = 0.0f;
        if (w > 0) {
            bar_sync_n(1 + w, 64);
            o = xo[w][lane];
            kvn = xk_[w][lane];
        }
        if (next) {
#pragma unroll
            for (int r = 0; r < kDnPart; r++) {
                o = __fadd_rn(o, po[r]);
                kvn = __fadd_rn(kvn, pk[r]);
            }
        } else {
#pragma unroll
            for (int r = 0; r < kDnPart; r++) o = __fadd_rn(o, po[r]);
        }
        if (w < kDnParts - 1) {
            xo[w + 1][lane] = o;
            xk_[w + 1][lane] = kvn;
            bar_arrive_n(2 + w, 64);
        } else {
            if (next) sdelta[lane] = __fmul_rn(__fadd_rn(sv[t + 1][lane], -kvn), sbeta[t + 1]);
#pragma unroll
            for (int r = 0; r < kDnCl; r++) st_dsmem(&so[t][col], (uint32_t)r, o);   // to every CTA
        }
        if (logged && t > 0 && w == 0) {   // log row t: k, delta per column, decay
            float *u = L.upd + (((size_t)wr * d.cap + t) * d.nv + h) * logw;
            u[kDK + col] = delta;
            u[col] = sk[t][col];
            if (col == 0) u[kDK + kDV] = sdec[t];
        }
    }
    // every CTA's output columns in every CTA (no shared memory of a peer is touched after this)
    cluster_arrive();
    cluster_wait();
    // ---- gated RMSNorm over the 128 outputs, then A8 of this CTA's 32-column block
    for (int u0 = w * 8; u0 < n; u0 += kDnParts * 8) {
        const int u = u0 + (lane >> 2), l = lane & 3;
        const bool act = u < n;
        const float *vec = so[act ? u : 0];
        float cs = 0.0f;
        if (act) {
#pragma unroll 32
            for (int i = l; i < kDV; i += 4) cs = madd(cs, vec[i], vec[i]);
        }
        const int base = lane & ~3;
        const float c0 = __shfl_sync(0xffffffffu, cs, base), c1 = __shfl_sync(0xffffffffu, cs, base + 1);
        const float c2 = __shfl_sync(0xffffffffu, cs, base + 2), c3 = __shfl_sync(0xffffffffu, cs, base + 3);
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
        if (act && l == 0) srn[u] = inv_sqrt_ref(__fadd_rn(__fdiv_rn(ss, (float)kDV), d.eps));
    }
    __syncthreads();
    {
        const int nbo = out.cols >> 5, gcol = h * kDV + col;
        const float nw = L.norm_w[col];
#pragma unroll
        for (int q = 0; q < NT; q++) {
            const int t = w + q * kDnParts;
            if (t < n) {
                float v = __fmul_rn(__fmul_rn(so[t][col], srn[t]), nw);
                v = __fmul_rn(v, pf_silu(zt[q]));
                quant_block_warp(v, lane, out.q + (size_t)t * out.cols + (gcol & ~31), out.d + (size_t)t * nbo + (gcol >> 5),
                                 out.fs + (size_t)t * nbo + (gcol >> 5));
            }
        }
    }
}

// Gated DeltaNet layer of a prefill chunk, rows 0..n-1 of y (any n), in three kernels, with no
// deferred commit to replay and nothing logged (the caller flushes a pending commit first). The
// per-element arithmetic is k_deltanet2's (same citations); the work is split by its shape:
//   k_deltanet_prep  conv + SiLU of every q / k / v channel, the L2 norms and the gates: the conv
//                    is a filter over the inputs (rows b - 3 .. b), so every 16-row block of every
//                    head is independent (grid heads x blocks); one record per (row, head).
//   k_deltanet_rows  the recurrence, sequential over the rows: one CTA per key head, thread j owns
//                    state column j with all of its kDK rows in registers for the whole chunk, so
//                    a token's update, its output dot product and the next token's kv dot product
//                    are one sweep over the rows with the two ordered add chains (rows 0..kDK-1 in
//                    order, kern_lin.c) interleaved and no partial sum crossing threads; the
//                    records stream in by bulk copies, two 16-row blocks in flight.
//   k_deltanet_post  the gated RMSNorm over a row's 128 outputs and the A8 of the result (grid
//                    rows x heads).
// The elementwise products take two rows per packed f32x2 instruction (each lane rounds as the
// scalar operation), except the k * delta products: ptxas contracts a packed multiply that
// feeds a packed add into one fused multiply-add (one rounding instead of two; measured on
// B200 with CUDA 12.9, --fmad=false and explicit .rn alike), so those stay scalar __fmul_rn.
// The decay of a block's first token is applied in a sweep of its own instead of inside the
// previous token's: per element the same operations in the same order.
constexpr int kDnBlk = 16;
constexpr int kDnCh = kDK + kDK + kDV;          // channels of one head: q ++ k ++ v
constexpr int kDnRec = kDnCh + 4;               // record: q, k (L2-normed), v (conv), beta, decay, 2 pad

// st == nullptr: one chunk of n rows (grid heads x 16-row blocks); else one pass of up to 16 rows
// per sequence of a batch (grid heads x sequences; sequence i's rows at st[i].row0, its states
// at the batch's per-sequence strides).
template <int KC>
__global__ void __launch_bounds__(kDnCh) k_deltanet_prep(LinLayer L, LinDims d, const float *y, int n, float *recs,
                                                         const Step *st) {
    constexpr int S = KC - 1;
    const int h = blockIdx.x, c = threadIdx.x, w = c >> 5, lane = c & 31;
    int b0 = blockIdx.y * kDnBlk, base = b0, nb = n - b0 < kDnBlk ? n - b0 : kDnBlk;
    if (st) {   // written between passes only, so read before pdl_wait
        st += blockIdx.y;
        L.conv_state += blockIdx.y * d.ss_conv;
        b0 = 0;
        base = ld_early_s32(&st->row0);
        nb = ld_early_s32(&st->n);
        nb = nb < kDnBlk ? nb : kDnBlk;
    }
    const int C = d.C;
    const int ch = c < kDK ? h * kDK + c : c < 2 * kDK ? d.kd + h * kDK + (c - kDK) : 2 * d.kd + h * kDV + (c - 2 * kDK);
    // taps, and for the chunk's first block the conv state (written by this layer's DeltaNet of
    // an earlier pass, before this kernel's predecessor): requested before pdl_wait
    ConvCh<KC> cv;
    cv.c = ch;
#pragma unroll
    for (int r = 0; r < KC; r++) cv.w[r] = ld_early(L.conv_w + (size_t)ch * KC + r);
#pragma unroll
    for (int r = 0; r < S; r++) cv.st[r] = b0 == 0 ? ld_early(L.conv_state + (size_t)r * C + ch) : 0.0f;
    pdl_wait();
    pdl_trigger();
    if (nb <= 0) return;
    if (b0 > 0) {   // a later block: the state is the chunk's own three inputs before it
#pragma unroll
        for (int r = 0; r < S; r++) cv.st[r] = y[(size_t)(base - S + r) * d.ldy + ch];
    }
    __shared__ __align__(16) float sx[kDnBlk][kDnCh + 4];
    __shared__ float sg[kDnBlk][2];
    float xin[kDnBlk];
#pragma unroll
    for (int t = 0; t < kDnBlk; t++) xin[t] = t < nb ? ld_early(y + (size_t)(base + t) * d.ldy + ch) : 0.0f;
#pragma unroll
    for (int t = 0; t < kDnBlk; t++)
        if (t < nb) sx[t][c] = conv_step(cv, xin[t]);
    if (c < nb) {   // gates of row base + c
        const float *yr = y + (size_t)(base + c) * d.ldy;
        const float gb = yr[C + d.vd + h], ga = yr[C + d.vd + d.nv + h];
        sg[c][0] = __fdiv_rn(1.0f, __fadd_rn(1.0f, glibc_expf(-gb)));
        const float xs = __fadd_rn(ga, L.dt_bias[h]);
        const float sp = xs > 20.0f ? xs : glibc_log1pf(glibc_expf(xs));
        sg[c][1] = glibc_expf(__fmul_rn(L.A[h], sp));
    }
    __syncthreads();
    // L2 norm of q and k: 4 lanes per (row, vector)
    if (w < 4) {
        const float qscale = inv_sqrt_ref((float)kDK);
        const int u = w * 8 + (lane >> 2), l = lane & 3;
        const bool act = u < 2 * nb;
        float *vec = act ? &sx[u >> 1][(u & 1) * kDK] : &sx[0][0];
        float cs = 0.0f;
        if (act) {
#pragma unroll 32
            for (int i = l; i < kDK; i += 4) cs = madd(cs, vec[i], vec[i]);
        }
        const int base = lane & ~3;
        const float c0 = __shfl_sync(0xffffffffu, cs, base), c1 = __shfl_sync(0xffffffffu, cs, base + 1);
        const float c2 = __shfl_sync(0xffffffffu, cs, base + 2), c3 = __shfl_sync(0xffffffffu, cs, base + 3);
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
        const float r = inv_sqrt_ref(__fadd_rn(ss, 1e-6f));
        __syncwarp();
        if (act) {
            const float sc = (u & 1) ? 1.0f : qscale;
            for (int i = l; i < kDK; i += 4) vec[i] = __fmul_rn(__fmul_rn(vec[i], r), sc);
        }
    }
    static_assert(2 * kDnBlk <= 4 * 8, "one pass of four warps covers the block's vectors");
    __syncthreads();
    for (int t = 0; t < nb; t++) {
        float *rec = recs + ((size_t)(base + t) * d.nk + h) * kDnRec;
        rec[c] = sx[t][c];
        if (c < 2) rec[kDnCh + c] = sg[t][c];
    }
}

__global__ void __launch_bounds__(kDV, 1) k_deltanet_rows(LinLayer L, LinDims d, const float *y, int n,
                                                          const float *recs, float *o_rows, int *status,
                                                          Step *st) {
    constexpr int KC = 4, S = KC - 1, NP = kDK / 2;
    const int h = blockIdx.x, j = threadIdx.x;
    const int C = d.C;
    int base = 0;
    if (st) {   // one sequence of a batch pass: its rows, states and status word
        st += blockIdx.y;
        L.conv_state += blockIdx.y * d.ss_conv;
        L.rec += blockIdx.y * d.ss_rec;
        n = ld_early_s32(&st->n);
        base = ld_early_s32(&st->row0);
        status = &st->status;
        if (ld_early_s32(&st->logged) || ld_early_s32(&st->pend_keep) > 0 || ld_early_s32(&st->pend_conv) > 0) {
            // a verify pass or a deferred commit: not this kernel's (the engine never sends one)
            pdl_wait();
            pdl_trigger();
            if (j == 0) st->status = -92;
            return;
        }
    }
    // the state column: written only by this layer's recurrence in an earlier chunk (a sequence
    // with no rows in this pass leaves it alone)
    float *rec = L.rec + (size_t)h * kDK * kDV + j;
    float2 Sc[NP];   // rows (2 m, 2 m + 1) of column j
#pragma unroll
    for (int m = 0; m < NP; m++) Sc[m] = make_float2(0.0f, 0.0f);
    if (n > 0) {
#pragma unroll
        for (int m = 0; m < NP; m++)
            Sc[m] = make_float2(ld_early(rec + (size_t)(2 * m) * kDV), ld_early(rec + (size_t)(2 * m + 1) * kDV));
    }
    extern __shared__ __align__(16) float dnb[];   // [2][kDnBlk][kDnRec]: two blocks of records
    __shared__ __align__(8) uint64_t bar[2];
    if (j == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    if (n <= 0) return;
    const int nblk = (n + kDnBlk - 1) / kDnBlk;
    auto issue = [&](int b) {   // thread 0: block b's records into buffer b % 2
        const int b0 = b * kDnBlk, nb = n - b0 < kDnBlk ? n - b0 : kDnBlk;
        float *dst = dnb + (size_t)(b & 1) * kDnBlk * kDnRec;
        mbar_arrive_expect(&bar[b & 1], (uint32_t)(nb * kDnRec * 4));
        for (int t = 0; t < nb; t++)
            bulk_g2s(dst + (size_t)t * kDnRec, recs + ((size_t)(base + b0 + t) * d.nk + h) * kDnRec, kDnRec * 4,
                     &bar[b & 1]);
    };
    if (j == 0) {
        issue(0);
        if (nblk > 1) issue(1);
    }
    bool ok = true;
    for (int b = 0; b < nblk; b++) {
        const int b0 = b * kDnBlk, nb = n - b0 < kDnBlk ? n - b0 : kDnBlk;
        if (!mbar_wait(&bar[b & 1], (uint32_t)(b >> 1) & 1u)) {   // timed out: reported, no hang
            ok = false;
            break;
        }
        const float *blk = dnb + (size_t)(b & 1) * kDnBlk * kDnRec;
        // the block's first decay and kv (rows in order)
        float kv = 0.0f;
        {
            const float dec = blk[kDnCh + 1];
            const float2 dec2 = make_float2(dec, dec);
            const float4 *k4 = reinterpret_cast<const float4 *>(blk + kDK);
#pragma unroll
            for (int m = 0; m < NP; m += 2) {
                const float4 kk = k4[m / 2];
                Sc[m] = __fmul2_rn(Sc[m], dec2);
                Sc[m + 1] = __fmul2_rn(Sc[m + 1], dec2);
                const float2 p0 = __fmul2_rn(Sc[m], make_float2(kk.x, kk.y));
                const float2 p1 = __fmul2_rn(Sc[m + 1], make_float2(kk.z, kk.w));
                kv = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(kv, p0.x), p0.y), p1.x), p1.y);
            }
        }
        // tokens: S += k delta, o = S.q; then S *= decay of the next token, its kv = S.k
        for (int t = 0; t < nb; t++) {
            const float *r = blk + (size_t)t * kDnRec;
            const float delta = __fmul_rn(__fadd_rn(r[2 * kDK + j], -kv), r[kDnCh]);
            const float4 *q4 = reinterpret_cast<const float4 *>(r);
            const float4 *k4 = reinterpret_cast<const float4 *>(r + kDK);
            float o = 0.0f, kvn = 0.0f;
            if (t + 1 < nb) {
                const float *rn = r + kDnRec;
                const float dn = rn[kDnCh + 1];
                const float2 dn2 = make_float2(dn, dn);
                const float4 *n4 = reinterpret_cast<const float4 *>(rn + kDK);
#pragma unroll
                for (int m = 0; m < NP; m += 2) {
                    const float4 kk = k4[m / 2], qq = q4[m / 2], nn = n4[m / 2];
                    float2 s0 = __fadd2_rn(Sc[m], make_float2(__fmul_rn(kk.x, delta), __fmul_rn(kk.y, delta)));
                    float2 s1 = __fadd2_rn(Sc[m + 1], make_float2(__fmul_rn(kk.z, delta), __fmul_rn(kk.w, delta)));
                    const float2 p0 = __fmul2_rn(s0, make_float2(qq.x, qq.y));
                    const float2 p1 = __fmul2_rn(s1, make_float2(qq.z, qq.w));
                    s0 = __fmul2_rn(s0, dn2);
                    s1 = __fmul2_rn(s1, dn2);
                    const float2 r0 = __fmul2_rn(s0, make_float2(nn.x, nn.y));
                    const float2 r1 = __fmul2_rn(s1, make_float2(nn.z, nn.w));
                    o = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(o, p0.x), p0.y), p1.x), p1.y);
                    kvn = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(kvn, r0.x), r0.y), r1.x), r1.y);
                    Sc[m] = s0;
                    Sc[m + 1] = s1;
                }
            } else {
#pragma unroll
                for (int m = 0; m < NP; m += 2) {
                    const float4 kk = k4[m / 2], qq = q4[m / 2];
                    const float2 s0 = __fadd2_rn(Sc[m], make_float2(__fmul_rn(kk.x, delta), __fmul_rn(kk.y, delta)));
                    const float2 s1 = __fadd2_rn(Sc[m + 1], make_float2(__fmul_rn(kk.z, delta), __fmul_rn(kk.w, delta)));
                    const float2 p0 = __fmul2_rn(s0, make_float2(qq.x, qq.y));
                    const float2 p1 = __fmul2_rn(s1, make_float2(qq.z, qq.w));
                    o = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(o, p0.x), p0.y), p1.x), p1.y);
                    Sc[m] = s0;
                    Sc[m + 1] = s1;
                }
            }
            o_rows[(size_t)(base + b0 + t) * d.vd + h * kDV + j] = o;
            kv = kvn;
        }
        __syncthreads();   // every thread is done with buffer b % 2 before it is refilled
        if (j == 0 && b + 2 < nblk) issue(b + 2);
    }
    if (!ok) {   // let the copies in flight land (a second bounded wait) before shared memory goes
        if (j == 0 && status) *status = -90;
        mbar_wait(&bar[0], 0);
        mbar_wait(&bar[1], 0);
        return;
    }
#pragma unroll
    for (int m = 0; m < NP; m++) {
        rec[(size_t)(2 * m) * kDV] = Sc[m].x;
        rec[(size_t)(2 * m + 1) * kDV] = Sc[m].y;
    }
    // conv states: the last three inputs of [old state, rows 0..n-1] for this thread's channels
    const int chs[3] = {h * kDK + j, d.kd + h * kDK + j, 2 * d.kd + h * kDV + j};
#pragma unroll
    for (int q = 0; q < 3; q++) {
        float v[S];
#pragma unroll
        for (int r = 0; r < S; r++) {
            const int i = n + r;   // index into [old 0..S-1, row 0, row 1, ...]
            v[r] = i < S ? L.conv_state[(size_t)i * C + chs[q]] : y[(size_t)(base + i - S) * d.ldy + chs[q]];
        }
#pragma unroll
        for (int r = 0; r < S; r++) L.conv_state[(size_t)r * C + chs[q]] = v[r];
    }
}

// The gated RMSNorm of one row's 128 outputs of one head, then A8 (grid rows x heads).
__global__ void __launch_bounds__(kDV) k_deltanet_post(LinLayer L, LinDims d, const float *y, const float *o_rows,
                                                       Act out) {
    const int v = blockIdx.x, h = blockIdx.y, j = threadIdx.x, lane = j & 31;
    const float nw = L.norm_w[j];
    pdl_wait();
    pdl_trigger();
    __shared__ float so[kDV];
    __shared__ float srn;
    const int col = h * kDV + j;
    so[j] = o_rows[(size_t)v * d.vd + col];
    const float z = y[(size_t)v * d.ldy + d.C + col];
    __syncthreads();
    if (j < 32) {
        const int l = lane & 3;
        float cs = 0.0f;
        if (lane < 4) {
#pragma unroll 32
            for (int i = l; i < kDV; i += 4) cs = madd(cs, so[i], so[i]);
        }
        const float c0 = __shfl_sync(0xffffffffu, cs, 0), c1 = __shfl_sync(0xffffffffu, cs, 1);
        const float c2 = __shfl_sync(0xffffffffu, cs, 2), c3 = __shfl_sync(0xffffffffu, cs, 3);
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3)), 0.0f);
        if (lane == 0) srn = inv_sqrt_ref(__fadd_rn(__fdiv_rn(ss, (float)kDV), d.eps));
    }
    __syncthreads();
    float x = __fmul_rn(__fmul_rn(so[j], srn), nw);
    x = __fmul_rn(x, pf_silu(z));
    const int nbo = out.cols >> 5;
    quant_block_warp(x, lane, out.q + (size_t)v * out.cols + (col & ~31), out.d + (size_t)v * nbo + (col >> 5),
                     out.fs + (size_t)v * nbo + (col >> 5));
}


// ------------------------------------------------------------------ MTP draft head
// The Qwen3.5 MTP head (engine/src/mtp.c:60-100, semantics engine/src/mtp.h): row t at position
// pos0 + t takes a final-normed hidden h[t] and the token that follows that position;
//   u = fc([rmsnorm(embed(tok), norm_emb) | rmsnorm(h, norm_hid)]), one full-attention decoder
//   block with its own KV cache, m = rmsnorm(u, norm_out), logits = head[0:nv) m.
// The block and the head reuse the main model's kernels; these kernels add the input rows, the
// normed-row export, and the hand-offs between the passes of a verify round (draft chain, then
// the pass over the accepted rows that leaves the next round's first draft).

// one dequantised row element of a Q4K embedding (kern_get_row_q, engine/src/kern_act.c:53-86)
__device__ __forceinline__ float embed_val(const Mat &E, int tok, int c) {
    const int panel = tok >> 5, r = tok & 31;
    const int sb = c >> 8, k = (c >> 5) & 7, j = c & 31;
    const uint8_t *u = E.w + ((size_t)panel * E.nsb + sb) * kUnitBytes + r * 16;
    const uint4 sc = *reinterpret_cast<const uint4 *>(u);
    const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
    const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
    const float dd = __fmul_rn(half_bits_to_float((uint32_t)(A >> 48)), (float)(uint32_t)((A >> (6 * k)) & 63u));
    const float mm = __fmul_rn(half_bits_to_float((uint32_t)(B >> 48)), (float)(uint32_t)((B >> (6 * k)) & 63u));
    const uint8_t byte = u[512 * (k + 1) + (j & 15)];
    const float q = (float)(j < 16 ? (byte & 15) : (byte >> 4));
    return __fadd_rn(__fmul_rn(dd, q), -mm);
}

// pf_norm_rows without quantisation: out [n][H] = (x r) w, r = 1 / sqrtf(sumsq / H + eps)
__global__ void k_norm_rows(const float *x, const float *w, int H, float eps, const Step *st, float *out) {
    pdl_wait();
    pdl_trigger();
    st += blockIdx.y;   // the sub-pass of a multi-pass chunk (row r = its row0 + v)
    if ((int)blockIdx.x >= st->n) return;
    const int v = st->row0 + blockIdx.x;
    extern __shared__ float xr[];   // [H]
    __shared__ float rr;
    for (int i = threadIdx.x; i < H; i += blockDim.x) xr[i] = x[(size_t)v * H + i];
    __syncthreads();
    if (threadIdx.x < 32) {
        const float s = sumsq_ref(xr, H);
        if (threadIdx.x == 0) rr = inv_sqrt_ref(__fadd_rn(__fdiv_rn(s, (float)H), eps));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(size_t)v * H + i] = __fmul_rn(__fmul_rn(xr[i], rr), w[i]);
}

// MTP input rows (mtp.c:76-83): [rmsnorm(embed(tok)) | rmsnorm(h)] (2H columns), A8-quantised
// for the fc projection. h [n][H] rows, tokens from the pass's step block.
__global__ void k_mtp_input(Mat E, const float *h, const Step *ms, const float *w_emb, const float *w_hid,
                            int H, float eps, Act out) {
    pdl_wait();
    pdl_trigger();
    ms += blockIdx.y;   // the sub-pass of a multi-pass chunk (row r = its row0 + blockIdx.x)
    if ((int)blockIdx.x >= ms->n) return;
    const int v = ms->row0 + blockIdx.x;
    extern __shared__ float cat[];   // [2H]: embedding row, hidden row
    __shared__ float r2[2];
    int tok = ms->tokens[blockIdx.x];
    if (tok < 0 || tok >= E.rows) tok = 0;   // ids come from the argmax of this head
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        cat[c] = embed_val(E, tok, c);
        cat[H + c] = h[(size_t)v * H + c];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (warp < 2) {
        const float s = sumsq_ref(cat + warp * H, H);
        if (lane == 0) r2[warp] = inv_sqrt_ref(__fadd_rn(__fdiv_rn(s, (float)H), eps));
    }
    __syncthreads();
    const int nb = (2 * H) >> 5;
    for (int b = warp; b < nb; b += nw) {
        const int i = b * 32 + lane;
        const float y = i < H ? __fmul_rn(__fmul_rn(cat[i], r2[0]), w_emb[i])
                              : __fmul_rn(__fmul_rn(cat[i], r2[1]), w_hid[i - H]);
        quant_block_warp(y, lane, out.q + (size_t)v * out.cols + b * 32, out.d + (size_t)v * nb + b,
                         out.fs + (size_t)v * nb + b);
    }
}

// Chain step s of a verify round (spec.c:300-321): draft s + 1 from (m of draft s, draft s) at
// position P - 1 + s; runs only while s < ke (verify rows - 1).
__global__ void k_mtp_chain_set(Step *st, Step *ms, int s) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    const int n = st->n;
    int run = (n > 0 && !st->use_ng && s < n - 1) ? 1 : 0;
    // adaptive (spec.c:310): draft s + 1 only while draft s's top-1 probability >= 0.6
    if (run && st->adaptive && (st->chain_stop || !(st->conf >= 0.6f))) {
        run = 0;
        if (!st->chain_stop) {
            st->chain_stop = 1;
            st->n = s + 1;   // verify cur and drafts 1..s
        }
    }
    ms->n = run;
    ms->pos0 = st->pos0 - 1 + s;
    ms->tokens[0] = st->tokens[s];
    ms->logged = 0;
}
__global__ void k_mtp_chain_take(Step *st, const Step *ms, int s, const float *mrows, float *mcur, int H) {
    pdl_wait();
    pdl_trigger();
    if (ms->n <= 0) return;
    if (threadIdx.x == 0) st->tokens[s + 1] = ms->argmax[0];
    for (int i = threadIdx.x; i < H; i += blockDim.x) mcur[i] = mrows[i];
}
// The pass over the rows the last verify committed (spec.c:369-374, mtp_pending): their main
// hiddens, the tokens that followed them, their positions.
__global__ void k_mtp_pending_set(const Step *st, Step *ms) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    const int e = st->last_e;
    ms->n = e;
    ms->pos0 = st->last_pos;
    for (int t = 0; t < e && t < kMaxRows; t++) ms->tokens[t] = st->last_tok[t];
    ms->logged = 0;
}
__device__ void plan_round(Step *st, const int *greedy);   // below, with the generation control
__device__ void ad_record(Step *st, int n, int e);

// Its last row drafts the next round's first token; its m seeds the next chain.
__global__ void k_mtp_pending_take(Step *st, const Step *ms, const float *mrows, float *mcur, int H) {
    pdl_wait();
    pdl_trigger();
    const int n = ms->n;
    if (n <= 0) return;
    if (threadIdx.x == 0) {
        st->mtp_d1 = ms->argmax[n - 1];
        if (!st->done && st->logged) {   // verify rounds: the next round
            if (st->adaptive) ad_record(st, st->last_n, st->last_e);
            plan_round(st, nullptr);
        }
    }
    for (int i = threadIdx.x; i < H; i += blockDim.x) mcur[i] = mrows[(size_t)(n - 1) * H + i];
}
// Adaptive speculation: timestamps of the round's phases (%globaltimer, nanoseconds).
__global__ void k_stamp(Step *st, int idx) {
    pdl_wait();
    pdl_trigger();
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    st->t_stamp[idx] = t;
}
// Top-1 probability of the newest MTP draft (top1_prob, spec.c:89-92): 1 / sum exp(l - max)
// over the draft vocabulary, for the chain rule of the adaptive policy. The max is exact; the
// sum is a parallel tree (the reference's 4-lane order would take ~60 K dependent adds), so a
// decision can differ from the reference's only where the probability lies within rounding
// of the 0.6 threshold.
__global__ void __launch_bounds__(1024) k_conf(const float *logits, int ld, int nv, const Step *ms, Step *st) {
    pdl_wait();
    pdl_trigger();
    const int n = ms->n;
    if (n <= 0) return;
    const float *l = logits + (size_t)(n - 1) * ld;
    __shared__ float red[32];
    __shared__ float s_m;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) m = fmaxf(m, l[i]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        float v = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
        for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) s_m = v;
    }
    __syncthreads();
    const float mx = s_m;
    float sum = 0.0f;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) sum = __fadd_rn(sum, pf_expf(__fadd_rn(l[i], -mx)));
    for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    __syncthreads();
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (warp == 0) {
        float v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) st->conf = v > 0.0f ? __fdiv_rn(1.0f, v) : 0.0f;
    }
}

// Prefill: the prompt's last row pairs with the first generated token (spec.c:186-190).
__global__ void k_mtp_prefill_fix(const Step *st, Step *ms) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0 && ms->n > 0 && st->n > 0) ms->tokens[ms->n - 1] = st->argmax[st->n - 1];
}

// ------------------------------------------------------------------ generation control
// splitmix64 output function and the synthetic drafter of the benchmark: the draft for output
// index j is, with probability p24 / 2^24, the target's greedy token greedy[j], else a uniform
// token (the same function as the CPU harness, oracle/ref_spec.c).
__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
__device__ __forceinline__ int synth_draft(unsigned long long seed, long long j, unsigned p24,
                                           int vocab, int greedy_j) {
    const unsigned long long h = mix64(seed ^ mix64((unsigned long long)j));
    if ((unsigned)(h >> 40) < p24) return greedy_j;
    return (int)(mix64(h) % (unsigned long long)vocab);
}

// One emitted token (spec.c emit, engine/src/spec.c:206-215): returns 1 when generation stops.
__device__ __forceinline__ int emit_tok(Step *st, int *out, int tok) {
    out[st->count++] = tok;
    int stop = st->count >= st->n_max;
    if (tok == st->eos) stop = 1;
    for (int i = 0; i < st->n_stop && !stop; i++) stop = tok == st->stop_ids[i];
    return stop;
}

// ---- prompt lookup (engine/src/ngram.c, restated): one direct-mapped hash table per n-gram
// length 2..4 maps an n-gram of the token history to the position where it most recently
// ended (+1); new positions are indexed lazily by the next lookup; every hit is verified
// against the history, so a collision can only lose a match. The hash (FNV-1 offset basis
// mixed with the length, golden-ratio multiplier) and the table size (2^bits >= 2 x capacity,
// 10 <= bits <= 24) are the reference's, so its drafts and ours coincide.
constexpr int kNgMin = 2, kNgMax = 4, kNgExt = 32;
constexpr int kNgTrust = 16, kNgAsk = 4, kNgShort = 3;   // spec.h PF_NG_TRUST / ASK / SHORT

__device__ __forceinline__ uint32_t ng_hash(const int *t, int n, int bits) {
    uint32_t h = 0x811C9DC5u ^ (uint32_t)n;
    for (int i = 0; i < n; i++) h = (h ^ (uint32_t)t[i]) * 0x9E3779B1u;
    return h >> (32 - bits);
}
// append a token (past the capacity it is dropped: drafting only gets weaker)
__device__ __forceinline__ void ng_push(Step *st, int tok) {
    if (st->hist && st->hist_n < st->hist_cap) st->hist[st->hist_n++] = tok;
}
// index the n-grams that end at positions [hist_idx, upto)
__device__ void ng_index(Step *st, int upto) {
    for (int q = st->hist_idx; q < upto; q++)
        for (int n = kNgMin; n <= kNgMax && n <= q + 1; n++)
            st->ng_tab[((size_t)(n - kNgMin) << st->ng_bits) + ng_hash(st->hist + q - n + 1, n, st->ng_bits)] = q + 1;
    if (upto > st->hist_idx) st->hist_idx = upto;
}
// up to max tokens that followed the most recent earlier occurrence of the longest matching
// tail n-gram; *match = how far back the two occurrences agree (n .. kNgExt)
__device__ int ng_draft(Step *st, int *out, int max, int *match) {
    const int n = st->hist_n;
    *match = 0;
    if (!st->hist || max <= 0 || n < kNgMin + 1) return 0;
    // index every position but the newest: a match for the tail must lie strictly earlier
    ng_index(st, n - 1);
    for (int k = kNgMax; k >= kNgMin; k--) {
        if (k > n - 1) continue;
        const int *tail = st->hist + n - k;
        const int q = st->ng_tab[((size_t)(k - kNgMin) << st->ng_bits) + ng_hash(tail, k, st->ng_bits)] - 1;
        if (q < k - 1 || q >= n - 1) continue;
        bool same = true;
        for (int i = 0; i < k && same; i++) same = st->hist[q - k + 1 + i] == tail[i];
        if (!same) continue;
        const int m = n - 1 - q < max ? n - 1 - q : max;
        for (int i = 0; i < m; i++) out[i] = st->hist[q + 1 + i];
        int e = k;
        while (e < kNgExt && q - e >= 0 && st->hist[q - e] == st->hist[n - 1 - e]) e++;
        *match = e;
        return m;
    }
    return 0;
}

// ---- adaptive policy (engine/src/spec_adapt.c, restated): EMA of verify-pass times per width,
// decayed tokens and seconds of the speculative rounds, plain mode when speculation measures
// >= 5 % slower than plain steps (or than any verify pass, the sure case), probes out of plain
// mode after 8, 16, .. 64 plain steps, each probe decided by its own 2 rounds.
__device__ __forceinline__ double ad_ema(double old, double x) { return old <= 0.0 ? x : old + 0.25 * (x - old); }

__device__ bool ad_plain_now(Step *st) {
    if (!st->ad_plain_mode) return false;
    if (st->ad_plain_run < st->ad_probe_after) return true;
    if (!st->ad_probing) {   // a probe starts
        st->ad_probing = 1;
        st->ad_n_spec = 0;
        st->ad_r_tok = st->ad_r_sec = 0.0;
    }
    return false;
}
__device__ void ad_plain(Step *st, double sec) {
    st->ad_t_plain = ad_ema(st->ad_t_plain, sec);
    if (st->ad_plain_mode) st->ad_plain_run++;
}
__device__ void ad_round(Step *st, int n, int emitted, double sec, double t_verify) {
    if (n < 2 || n > kMaxRows) return;
    st->ad_tv[n] = ad_ema(st->ad_tv[n], t_verify);
    st->ad_r_tok = 0.95 * st->ad_r_tok + emitted;
    st->ad_r_sec = 0.95 * st->ad_r_sec + sec;
    st->ad_n_spec++;
    double tv_min = 0.0;
    for (int i = 2; i <= kMaxRows; i++)
        if (st->ad_tv[i] > 0.0 && (tv_min <= 0.0 || st->ad_tv[i] < tv_min)) tv_min = st->ad_tv[i];
    double ts = 0.0;   // a plain step's seconds: measured, else extrapolated from widths 2 and 3
    if (st->ad_t_plain > 0.0) ts = st->ad_t_plain;
    else if (st->ad_tv[2] > 0.0 && st->ad_tv[3] > 0.0) {
        const double t = 2.0 * st->ad_tv[2] - st->ad_tv[3];
        ts = t > 0.5 * st->ad_tv[2] ? t : 0.5 * st->ad_tv[2];
    }
    const bool slow = st->ad_r_tok * tv_min < 0.95 * st->ad_r_sec ||
                      (ts > 0.0 && st->ad_r_tok * ts < 0.95 * st->ad_r_sec);
    if (st->ad_plain_mode) {   // a probe round
        if (st->ad_n_spec < 2) return;
        st->ad_probing = 0;
        st->ad_plain_mode = slow;
        st->ad_probe_after = !slow ? 8 : (st->ad_probe_after * 2 < 64 ? st->ad_probe_after * 2 : 64);
        st->ad_plain_run = 0;
        st->ad_n_spec = 0;
        if (slow) st->ad_r_tok = st->ad_r_sec = 0.0;
    } else if (slow && (st->ad_n_spec >= 8 || (ts > 0.0 && st->ad_tv[2] >= 1.5 * ts && st->ad_n_spec >= 2))) {
        st->ad_plain_mode = 1;
        st->ad_plain_run = 0;
        st->ad_probe_after = 8;
    }
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// the measurements of the round that just committed (n rows verified, e tokens emitted)
__device__ void ad_record(Step *st, int n, int e) {
    const unsigned long long t_end = globaltimer();
    const double sec = (double)(t_end - st->t_stamp[0]) * 1e-9;
    const double tv = (double)(st->t_stamp[2] - st->t_stamp[1]) * 1e-9;
    if (n <= 1) ad_plain(st, tv);   // a plain step: its forward pass
    else ad_round(st, n, e, sec, tv);
}

// Shape and drafts of the next round (spec.c:280-321): never draft past n_max or the context;
// the n-gram draft when the history's tail occurred before and the match is trusted
// (ngram_pick, spec.c:138-151: a match of >= PF_NG_TRUST tokens in full; a shorter one only
// without the MTP head, or when it extends >= PF_NG_ASK tokens and its first token is the MTP
// head's d1, and then at most PF_NG_SHORT tokens); otherwise k drafts of the drafter. With the
// MTP head this runs after the round's MTP pass, whose d1 it compares against.
__device__ void plan_round(Step *st, const int *greedy) {
    int left = st->n_max - st->count - 1;
    const int room = st->max_ctx - st->pos0 - 1;
    if (left > room) left = room;
    if (left < 0) {
        st->status = -5;   // PINFER_E_CTX_FULL
        st->done = 1;
        st->n = 0;
        return;
    }
    int d[kMaxRows];
    int ke = 0, use_ng = 0;
    st->chain_stop = 0;
    const bool plain = st->adaptive && ad_plain_now(st);   // spec.c:288
    if (!plain && st->ngram > 0 && left > 0) {
        int match = 0;
        const int mx = min(min(st->ngram, left), kMaxRows - 1);
        const int nd = ng_draft(st, d, mx, &match);
        if (nd > 0) {
            if (match >= kNgTrust) ke = nd;
            else if (st->k == 0) ke = nd < kNgShort ? nd : kNgShort;
            else if (match >= kNgAsk && d[0] == st->mtp_d1) ke = nd < kNgShort ? nd : kNgShort;
        }
        use_ng = ke > 0;
    }
    if (!use_ng) ke = plain ? 0 : (st->k < left ? st->k : left);
    st->use_ng = use_ng;
    st->tokens[0] = st->cur;
    if (use_ng) {
        for (int s = 1; s <= ke; s++) st->tokens[s] = d[s - 1];
    } else if (st->drafter == 1) {
        // MTP drafts: d1 from the last MTP pass; drafts 2..ke come from this round's chain
        if (ke >= 1) st->tokens[1] = st->mtp_d1;
    } else {
        for (int s = 1; s <= ke; s++) {
            const long long j = st->count - 1 + s;
            st->tokens[s] = synth_draft(st->seed, j, st->p24, st->vocab, greedy ? greedy[j] : 0);
        }
    }
    st->n = ke + 1;
    st->logged = 1;
}

// After the prefill pass: the first token is the argmax of the prompt's last row.
__global__ void k_gen_start(Step *st, const int *greedy, int *out) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    st += blockIdx.x;   // the sequence of a batch: its Step, greedy stream and output row
    if (greedy) greedy += (size_t)blockIdx.x * st->n_max;
    out += (size_t)blockIdx.x * st->n_max;
    const int n = st->n;
    st->cur = st->argmax[n - 1];
    st->pos0 += n;
    st->count = 0;
    st->done = 0;
    st->status = 0;
    st->last_e = 0;
    ng_push(st, st->cur);   // the history: fed tokens, then every emitted one
    if (emit_tok(st, out, st->cur)) {
        st->done = 1;
        st->n = 0;
        return;
    }
    plan_round(st, greedy);
}

// Greedy acceptance and commit of one verify pass (spec.c:337-351): the longest draft prefix
// that equals the model's argmax, plus the model's own next token; the e emitted tokens are
// committed (recurrent updates deferred, conv shifted at the next pass) and n_past advances
// by e (stale KV rows above it are overwritten later).
__global__ void k_accept(Step *st, const int *greedy, int *out) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    st += blockIdx.x;   // the sequence of a batch: its Step, greedy stream and output row
    if (greedy) greedy += (size_t)blockIdx.x * st->n_max;
    out += (size_t)blockIdx.x * st->n_max;
    const int n = st->n;
    if (n <= 0) {
        st->last_e = 0;
        return;
    }
    const int ke = n - 1;
    int vt[kMaxRows + 1];
    for (int i = 0; i < n; i++) vt[i] = st->tokens[i];
    int a = 0, g = st->argmax[0];
    while (a < ke && vt[a + 1] == g) {
        a++;
        g = st->argmax[a];
    }
    vt[a + 1] = g;
    int e = 0, done = 0;
    while (e <= a && !done) done = emit_tok(st, out, vt[++e]);
    st->last_pos = st->pos0;   // for the MTP pass over the committed rows
    st->last_e = e;
    st->last_n = n;
    for (int i = 0; i < e; i++) st->last_tok[i] = vt[i + 1];
    st->pend_keep = e - 1;   // pf_lin_commit (forward_lin.c:413-432)
    st->pend_conv = e;
    st->wr ^= 1;
    st->pos0 += e;
    st->cur = vt[e];
    for (int i = 1; i <= e; i++) ng_push(st, vt[i]);
    st->rounds++;
    st->drafted += ke;
    st->accepted += a;
    if (st->use_ng) {
        st->ng_rounds++;
        st->ng_drafted += ke;
        st->ng_accepted += a;
    }
    if (done) {
        st->done = 1;
        st->n = 0;
        return;
    }
    // with the MTP head the next round is planned after this round's MTP pass (its d1)
    if (st->drafter != 1) {
        if (st->adaptive) ad_record(st, n, e);
        plan_round(st, greedy);
    }
}

}  // namespace

// ------------------------------------------------------------------ launchers
namespace {
template <int NMAX>
size_t mv_smem() { return sizeof(MvSmem<NMAX>); }

int mv_grid(const Mat &W) {
    return W.npanels;   // one panel per CTA
}

template <int NMAX>
void matvec_t(const Mat &W, Act in, const Step *st, float *y, int ldy, int mode, cudaStream_t s) {
    const size_t sm = mv_smem<NMAX>();
    if (mode == 0) {
        launch_k(k_matvec<NMAX, 0>, mv_grid(W), kMvThreads, sm, s, W, in, st, y, ldy);
    } else {
        launch_k(k_matvec<NMAX, 1>, mv_grid(W), kMvThreads, sm, s, W, in, st, y, ldy);
    }
}
template <int NMAX>
void swiglu_t(const Mat &G, const Mat &U, Act in, const Step *st, Act out, cudaStream_t s) {
    const size_t sm = mv_smem<NMAX>();
    launch_k(k_matvec_swiglu<NMAX>, mv_grid(G), kMvThreads, sm, s, G, U, in, st, out);
}
template <int NMAX>
void head_t(const Mat &W, Act in, const Step *st, float *logits, int ld, unsigned long long *partial,
            int *nan0, cudaStream_t s) {
    const size_t sm = mv_smem<NMAX>();
    launch_k(k_matvec_head<NMAX>, mv_grid(W), kMvThreads, sm, s, W, in, st, logits, ld, partial, nan0);
}
}  // namespace

int num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

// The per-block shared memory opt-in limit of sm_100 (static + dynamic).
constexpr int kSmemOptin = 227 * 1024;

// The largest dynamic shared memory a kernel may launch with: the opt-in limit less its static
// __shared__ arrays.
template <class K>
int dyn_smem_limit(K kern) {
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, kern) != cudaSuccess) return 0;
    return kSmemOptin - (int)a.sharedSizeBytes;
}

// Allow the kernel the whole opt-in limit: the attribute only bounds what a launch may request,
// and contexts with different sizes (max_ctx) share the kernels, so it is never lowered.
// Every kernel also prefers the largest shared-memory carveout: the kernels of a round follow
// one another on the same SMs with programmatic dependent launch, and an SM whose carveout a
// starting kernel would have to change cannot take that kernel's CTAs until it drains, which
// defeats the early launch the weight prefetch relies on.
template <class K>
void max_carveout(K kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}
template <class K>
void raise_smem(K kern, size_t want = 0) {
    (void)want;
    const int lim = dyn_smem_limit(kern);
    if (lim > 0) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    max_carveout(kern);
}

template <int NMAX, bool NORM>
void head_t2(const Mat &W, Act in, NormIn nin, const Step *st, float *y, int ldy,
             unsigned long long *partial, int *nan0, int row_base, cudaStream_t s) {
    const int grid = std::min(2 * num_sms(), (W.npanels + kTallWarps - 1) / kTallWarps);
    launch_k(k_mv_head<NMAX, NORM>, std::max(grid, 1), kTallWarps * 32, tall_smem(W.cols, NMAX, NORM), s,
             W, in, nin, const_cast<Step *>(st), y, ldy, partial, nan0, row_base);
}

template <bool NORM>
void head_mma_t(const Mat &W, Act in, NormIn nin, const Step *st, float *y, int ldy,
                unsigned long long *partial, int *nan0, int row_base, cudaStream_t s,
                unsigned long long *fbest = nullptr, int *fctr = nullptr) {
    const int grid = std::min(2 * num_sms(), (W.npanels + kTallWarps - 1) / kTallWarps);
    launch_k(k_mv_head_mma<NORM>, std::max(grid, 1), kTallWarps * 32, head_mma_smem(W.cols, NORM), s, W, in, nin,
             const_cast<Step *>(st), y, ldy, partial, nan0, row_base, fbest, fctr);
}

template <int NMAX, int EPI, bool NORM, int PPC = 1>
bool panel_t(const Mat &W0, const Mat &W1, Act in, NormIn nin, const Step *st, float *y, int ldy,
             Act out, cudaStream_t s, const L2Prefetch &pf = L2Prefetch()) {
    const int nmat = EPI == 3 ? 2 : PPC;
    // passes of several rows: 16 warps, since the units phase is latency-bound and splits into
    // as many short per-warp sequences as the block allows (a unit's blocks over 2 or 4 warps);
    // one-row passes: 8 warps (16 for more than 8 units)
    const int nunit = W0.nsb * nmat, nw = (NMAX > 1 || nunit > 8) ? kPanelWarps : 8;
    const size_t sm = panel_smem(nunit, W0.cols, nmat, NMAX, NORM);
    // 16-byte row loads of the inputs (every engine buffer is 256-byte aligned, cols % 256 == 0)
    if (((uintptr_t)nin.x | (uintptr_t)nin.w | (uintptr_t)in.q | (uintptr_t)in.d | (uintptr_t)in.fs) & 15) return false;
    static const int lim = dyn_smem_limit(k_mv_panel<NMAX, EPI, NORM, PPC>);
    if (sm > (size_t)lim) return false;
    launch_k(k_mv_panel<NMAX, EPI, NORM, PPC>, (W0.npanels + PPC - 1) / PPC, nw * 32, sm, s, W0, W1, in, nin,
             const_cast<Step *>(st), y, ldy, out, pf);
    return true;
}

template <int EPI>
bool slice_t(const Mat &W, Act in, const Step *st, float *y, int ldy, cudaStream_t s) {
    const size_t sm = slice_smem(W.nsb, W.cols);
    static const int lim = dyn_smem_limit(k_mv_slice<EPI>);
    if (sm > (size_t)lim || (((uintptr_t)in.q | (uintptr_t)in.d | (uintptr_t)in.fs) & 15)) return false;
    launch_k(k_mv_slice<EPI>, W.npanels * (kPanelRows / kSliceRows), kSliceWarps * 32, sm, s, W, in,
             const_cast<Step *>(st), y, ldy);
    return true;
}

void launch_matvec(const Mat &W, Act in, const Step *st, float *y, int ldy, int mode, int nmax,
                   cudaStream_t s) {
    Act none;
    NormIn nn{};
    bool done = false;
    // long chains (64 or more blocks per row) on 8-row slices
    if (nmax > 1 && nmax <= 4 && W.cols >= 2048)
        done = mode ? slice_t<1>(W, in, st, y, ldy, s) : slice_t<0>(W, in, st, y, ldy, s);
    if (done) return;
    if (nmax <= 1) done = mode ? panel_t<1, 1, false>(W, W, in, nn, st, y, ldy, none, s) : panel_t<1, 0, false>(W, W, in, nn, st, y, ldy, none, s);
    else if (nmax <= 4) done = mode ? panel_t<4, 1, false>(W, W, in, nn, st, y, ldy, none, s) : panel_t<4, 0, false>(W, W, in, nn, st, y, ldy, none, s);
    if (!done) launch_matvec_chunked(W, in, st, y, ldy, mode, nmax, s);
}

void launch_matvec_norm(const Mat &W, const float *x, const float *w, float eps, const Step *st,
                        float *y, int ldy, int nmax, Act scratch, cudaStream_t s, const L2Prefetch &pf) {
    Act none;
    const NormIn nin{x, w, eps};
    bool done = false;
    if (nmax <= 1) done = panel_t<1, 0, true>(W, W, none, nin, st, y, ldy, none, s, pf);
    else if (nmax <= 4 && W.npanels > num_sms())   // two panels per CTA: one CTA per SM
        done = panel_t<4, 0, true, 2>(W, W, none, nin, st, y, ldy, none, s, pf);
    else if (nmax <= 4) done = panel_t<4, 0, true>(W, W, none, nin, st, y, ldy, none, s, pf);
    if (done) return;
    launch_norm_quant(x, w, W.cols, eps, st, scratch, s);
    launch_matvec_chunked(W, scratch, st, y, ldy, 0, nmax, s);
}

void launch_matvec_swiglu_norm(const Mat &G, const Mat &U, const float *x, const float *w, float eps,
                               const Step *st, Act out, int nmax, Act scratch, cudaStream_t s) {
    Act none;
    const NormIn nin{x, w, eps};
    bool done = false;
    if (nmax <= 1) done = panel_t<1, 3, true>(G, U, none, nin, st, nullptr, 0, out, s);
    else if (nmax <= 4) done = panel_t<4, 3, true>(G, U, none, nin, st, nullptr, 0, out, s);
    if (done) return;
    launch_norm_quant(x, w, G.cols, eps, st, scratch, s);
    if (nmax <= 1) swiglu_t<1>(G, U, scratch, st, out, s);
    else if (nmax <= 4) swiglu_t<4>(G, U, scratch, st, out, s);
    else if (nmax <= 8) swiglu_t<8>(G, U, scratch, st, out, s);
    else swiglu_t<16>(G, U, scratch, st, out, s);
}

void launch_matvec_head(const Mat &W, Act in, const Step *st, float *logits, int ld,
                        unsigned long long *partial, int *nan0, int nmax, cudaStream_t s, int row_base) {
    const NormIn nn{};
    if (nmax <= 4) head_mma_t<false>(W, in, nn, st, logits, ld, partial, nan0, row_base, s);
    else if (nmax <= 8) head_t2<8, false>(W, in, nn, st, logits, ld, partial, nan0, row_base, s);
    else head_t2<16, false>(W, in, nn, st, logits, ld, partial, nan0, row_base, s);
}

void launch_matvec_head_norm(const Mat &W, const float *x, const float *w, float eps, const Step *st,
                             float *logits, int ld, unsigned long long *partial, int *nan0, int nmax,
                             cudaStream_t s, int row_base, unsigned long long *fbest, int *fctr) {
    const NormIn nin{x, w, eps};
    const Act none;
    if (nmax <= 4) head_mma_t<true>(W, none, nin, st, logits, ld, partial, nan0, row_base, s, fbest, fctr);
    else if (nmax <= 8) head_t2<8, true>(W, none, nin, st, logits, ld, partial, nan0, row_base, s);
    else head_t2<16, true>(W, none, nin, st, logits, ld, partial, nan0, row_base, s);
}
// The first-generation kernel (chunked shared-memory chains, any shape) stays available for
// the kernel-level ABI's reference timing.
void launch_matvec_chunked(const Mat &W, Act in, const Step *st, float *y, int ldy, int mode,
                           int nmax, cudaStream_t s) {
    if (nmax <= 1) matvec_t<1>(W, in, st, y, ldy, mode, s);
    else if (nmax <= 4) matvec_t<4>(W, in, st, y, ldy, mode, s);
    else if (nmax <= 8) matvec_t<8>(W, in, st, y, ldy, mode, s);
    else matvec_t<16>(W, in, st, y, ldy, mode, s);
}
void launch_argmax_final(const unsigned long long *partial, const int *nan0, int npanels,
                         Step *st, cudaStream_t s, int nseq, int rps) {
    launch_k(k_argmax_final, dim3(rps, nseq), 256, 0, s, partial, nan0, npanels, st);
}
void launch_embed(const Mat &E, const Step *st, float *x, int H, cudaStream_t s, int nseq, int rps) {
    launch_k(k_embed, dim3(rps, nseq), 256, 0, s, E, st, x, H);
}
void launch_norm_quant(const float *x, const float *w, int H, float eps, const Step *st, Act out,
                       cudaStream_t s, int nseq, int rps) {
    launch_k(k_norm_quant, dim3(rps, nseq), 256, 2 * (size_t)H * sizeof(float), s, x, w, H, eps, st, out);
}
void launch_quant_act(const float *x, int n, int cols, Act out, cudaStream_t s) {
    const int warps = n * (cols / 32);
    launch_k(k_quant_act, (warps * 32 + 255) / 256, 256, 0, s, x, n, cols, out);
}
size_t deltanet_smem(int rep) {
    return sizeof(float) * ((size_t)kMaxRows * kDK * 2 + (size_t)kMaxRows * rep * kDV * 2 +
                            (size_t)kMaxRows * rep * 3 + (size_t)kMaxRows * kDK + kMaxRows + 8);
}
bool deltanet_batch_ok(const LinDims &d) {
    return d.rep == 1 && d.K == 4 && d.dk == kDK && d.dv == kDV && d.ldy % 4 == 0 && d.kd % 4 == 0 && d.C % 4 == 0 &&
           d.ss_rec % 4 == 0;
}
void launch_deltanet(const LinLayer &L, const LinDims &d, const float *y,
                     Step *st, Act out, cudaStream_t s, int nseq, int rps, int keep_max) {
    if (deltanet_batch_ok(d) && ((uintptr_t)y & 15) == 0 && ((uintptr_t)L.rec & 15) == 0) {
        const size_t sm = sizeof(float) * kDK * kDV;
        // a pass of rps rows follows a commit of at most rps rows of the same generation
        if (nseq == 1 && keep_max <= PINFER_SPEC_MAX_K) {   // one sequence: the 4-CTA cluster form
            const int pre = rps < kMaxRows ? rps : kMaxRows;
            if (pre <= 4)
                launch_k(k_deltanet3<4, 4, PINFER_SPEC_MAX_K>, dim3(d.nk * kDnCl, 1), kDnParts * 32, 0, s, L, d, y,
                         st, out, pre);
            else
                launch_k(k_deltanet3<4, kMaxRows, PINFER_SPEC_MAX_K>, dim3(d.nk * kDnCl, 1), kDnParts * 32, 0, s, L,
                         d, y, st, out, pre);
            return;
        }
        if (nseq > 1 && rps <= 4)
            launch_k(k_deltanet2<4, 4, 3>, dim3(d.nk, nseq), kDV, sm, s, L, d, y, st, out);
        else if (keep_max <= PINFER_SPEC_MAX_K)
            launch_k(k_deltanet2<4, kMaxRows, PINFER_SPEC_MAX_K>, dim3(d.nk, nseq), kDV, sm, s, L, d, y, st, out);
        else
            launch_k(k_deltanet2<4>, dim3(d.nk, nseq), kDV, sm, s, L, d, y, st, out);
        return;
    }
    if (nseq != 1) return;   // callers check deltanet_batch_ok first
    const size_t sm = deltanet_smem(d.rep);
    launch_k(k_deltanet, d.nk, kDV, sm, s, L, d, y, st, out);
}
size_t deltanet_rec_floats(const LinDims &d, int rows) { return (size_t)rows * d.nk * kDnRec; }
void launch_deltanet_rows(const LinLayer &L, const LinDims &d, const float *y, int n, float *recs, float *o_rows,
                          Act out, int *status, cudaStream_t s) {
    launch_k(k_deltanet_prep<4>, dim3(d.nk, (n + kDnBlk - 1) / kDnBlk), kDnCh, 0, s, L, d, y, n, recs,
             (const Step *)nullptr);
    launch_k(k_deltanet_rows, dim3(d.nk), kDV, sizeof(float) * 2 * kDnBlk * kDnRec, s, L, d, y, n,
             (const float *)recs, o_rows, status, (Step *)nullptr);
    launch_k(k_deltanet_post, dim3(n, d.nk), kDV, 0, s, L, d, y, (const float *)o_rows, out);
}
void launch_deltanet_rows_seqs(const LinLayer &L, const LinDims &d, const float *y, int R, Step *st, int nseq,
                               float *recs, float *o_rows, Act out, cudaStream_t s) {
    launch_k(k_deltanet_prep<4>, dim3(d.nk, nseq), kDnCh, 0, s, L, d, y, 0, recs, (const Step *)st);
    launch_k(k_deltanet_rows, dim3(d.nk, nseq), kDV, sizeof(float) * 2 * kDnBlk * kDnRec, s, L, d, y, 0,
             (const float *)recs, o_rows, (int *)nullptr, st);
    launch_k(k_deltanet_post, dim3(R, d.nk), kDV, 0, s, L, d, y, (const float *)o_rows, out);
}
void launch_attn_prep(const AttnLayer &L, const AttnDims &d, const float *y, float *qbuf,
                      const Step *st, cudaStream_t s, int nseq) {
    launch_k(k_attn_prep, dim3(d.rps * nseq, d.nq + d.nkv), d.hd, (size_t)d.hd * sizeof(float), s, L, d, y, qbuf, st);
}
bool attn4_ok(const AttnDims &d) {
    static const int attn4_lim = dyn_smem_limit(k_attn4);
    const int G = d.nkv > 0 ? d.nq / d.nkv : 0;
    return d.hd == kAttnHd && G > 0 && d.nq % d.nkv == 0 && G <= kAttnQ && kAttnQ % G == 0 &&
           attn4_smem(d.max_ctx) <= (size_t)attn4_lim;
}
bool attn5_ok(const AttnDims &d) {
    static const int attn5_lim = dyn_smem_limit(k_attn5<>);
    const int G = d.nkv > 0 ? d.nq / d.nkv : 0;
    return d.hd == kAttnHd && G > 0 && d.nq % d.nkv == 0 && G <= kAttnQ && kAttnQ % G == 0 &&
           attn5_smem(d.max_ctx) <= (size_t)attn5_lim;
}
bool attn_batch_ok(const AttnDims &d) {
    static const int attn3_lim = dyn_smem_limit(k_attn3);
    return d.hd == kAttnHd && attn3_smem(d.max_ctx) <= (size_t)attn3_lim;
}
void launch_attn(const AttnLayer &L, const AttnDims &d, const float *y, const float *qbuf,
                 const Step *st, Act out, cudaStream_t s, int nseq) {
    if (nseq > 1 && attn5_ok(d)) {   // one CTA per (sequence, KV group, rows): many in flight
        const int QR = kAttnQ / (d.nq / d.nkv), nch = (d.rps + QR - 1) / QR;
        launch_k(k_attn5<>, dim3(d.nkv * nch, nseq), kAttnHd, attn5_smem(d.max_ctx), s, L, d, y, qbuf, st, out);
        return;
    }
    if (nseq > 1 && attn4_ok(d)) {   // grouped queries share the K / V reads (one context: the
                                     // per-query clusters below have the shorter critical path)
        const int QR = kAttnQ / (d.nq / d.nkv), nch = (d.rps + QR - 1) / QR;
        launch_k(k_attn4, dim3(kAttnCL, d.nkv * nch, nseq), kAttnHd, attn4_smem(d.max_ctx), s, L, d, y, qbuf, st, out);
        return;
    }
    if (attn_batch_ok(d)) {
        launch_k(k_attn3, dim3(kAttnCL, d.nq, d.rps * nseq), kAttnHd, attn3_smem(d.max_ctx), s, L, d, y, qbuf, st, out);
        return;
    }
    if (nseq != 1) return;   // callers check attn_batch_ok first
    static const int attn2_lim = dyn_smem_limit(k_attn2);
    if (d.hd == kAttnHd && attn2_smem(d.max_ctx) <= (size_t)attn2_lim) {
        launch_k(k_attn2, dim3(kMaxRows, d.nq), kAttnHd, attn2_smem(d.max_ctx), s, L, d, y, qbuf, st, out);
        return;
    }
    const size_t sm = ((size_t)d.hd + d.max_ctx) * sizeof(float);
    launch_k(k_attn, dim3(kMaxRows, d.nq), d.hd, sm, s, L, d, y, qbuf, st, out);
}
void launch_attn_rows(const AttnLayer &L, const AttnDims &d, const float *y, const float *qbuf, const Step *st,
                      Act out, cudaStream_t s, int nseq) {
    static const int lim4 = dyn_smem_limit(k_attn5<4>), lim8 = dyn_smem_limit(k_attn5<8>);
    const int G = d.nkv > 0 && d.nq % d.nkv == 0 ? d.nq / d.nkv : 0;
    if (d.hd == kAttnHd && G == 4 && attn5_smem<4>(d.max_ctx) <= (size_t)lim4) {
        launch_k(k_attn5<4>, dim3(d.nkv * d.rps, nseq), kAttnHd, attn5_smem<4>(d.max_ctx), s, L, d, y, qbuf, st, out);
        return;
    }
    if (d.hd == kAttnHd && G == 8 && attn5_smem<8>(d.max_ctx) <= (size_t)lim8) {
        launch_k(k_attn5<8>, dim3(d.nkv * d.rps, nseq), kAttnHd, attn5_smem<8>(d.max_ctx), s, L, d, y, qbuf, st, out);
        return;
    }
    launch_attn(L, d, y, qbuf, st, out, s, nseq);
}
void launch_gen_start(Step *st, const int *greedy, int *out, cudaStream_t s, int nseq) {
    launch_k(k_gen_start, nseq, 32, 0, s, st, greedy, out);
}
void launch_accept(Step *st, const int *greedy, int *out, cudaStream_t s, int nseq) {
    launch_k(k_accept, nseq, 32, 0, s, st, greedy, out);
}
void launch_flush(const LinLayer *layers, int n_lin, const LinDims &d, Step *st, cudaStream_t s, int nseq) {
    FlushArgs fa;
    for (int i = 0; i < n_lin && i < kMaxLayers; i++) fa.layers[i] = layers[i];
    if (n_lin > 0) launch_k(k_flush, dim3(d.nk, n_lin, nseq), kDV, 0, s, fa, d, st);
    launch_k(k_clear_pending, nseq, 1, 0, s, st);
}
void launch_argmax_keys(const unsigned long long *partial, const int *nan0, int npanels, const Step *st,
                        unsigned long long *keys, cudaStream_t s, int kstride, int nseq, int rps) {
    launch_k(k_argmax_keys, dim3(rps, nseq), 256, 0, s, partial, nan0, npanels, st, keys, kstride);
}
void launch_keys_argmax(const unsigned long long *keys, Step *st, cudaStream_t s, int kstride, int nseq, int rps) {
    launch_k(k_keys_argmax, nseq, rps, 0, s, keys, st, kstride);
}
void launch_norm_rows(const float *x, const float *w, int H, float eps, const Step *st, float *out,
                      cudaStream_t s, int nseq) {
    launch_k(k_norm_rows, dim3(kMaxRows, nseq), 256, (size_t)H * sizeof(float), s, x, w, H, eps, st, out);
}
void launch_mtp_input(const Mat &E, const float *h, const Step *ms, const float *w_emb, const float *w_hid,
                      int H, float eps, Act out, cudaStream_t s, int nseq) {
    launch_k(k_mtp_input, dim3(kMaxRows, nseq), 256, 2 * (size_t)H * sizeof(float), s, E, h, ms, w_emb, w_hid, H, eps,
             out);
}
void launch_mtp_chain_set(Step *st, Step *ms, int step, cudaStream_t s) {
    launch_k(k_mtp_chain_set, 1, 32, 0, s, st, ms, step);
}
void launch_mtp_chain_take(Step *st, const Step *ms, int step, const float *mrows, float *mcur, int H,
                           cudaStream_t s) {
    launch_k(k_mtp_chain_take, 1, 256, 0, s, st, ms, step, mrows, mcur, H);
}
void launch_mtp_pending_set(const Step *st, Step *ms, cudaStream_t s) {
    launch_k(k_mtp_pending_set, 1, 32, 0, s, st, ms);
}
void launch_mtp_pending_take(Step *st, const Step *ms, const float *mrows, float *mcur, int H, cudaStream_t s) {
    launch_k(k_mtp_pending_take, 1, 256, 0, s, st, ms, mrows, mcur, H);
}
void launch_mtp_prefill_fix(const Step *st, Step *ms, cudaStream_t s) {
    launch_k(k_mtp_prefill_fix, 1, 32, 0, s, st, ms);
}
void launch_pass_end(Step *st, cudaStream_t s, int nseq) { launch_k(k_pass_end, nseq, 1, 0, s, st); }
void launch_set_pass(Step *st, int n, int pos0, int logged, const int *tokens, cudaStream_t s) {
    PassArgs a;
    a.n = n;
    a.pos0 = pos0;
    a.logged = logged;
    for (int i = 0; i < kMaxRows; i++) a.tokens[i] = i < n ? tokens[i] : 0;
    launch_k(k_set_pass, 1, 1, 0, s, st, a);
}
void launch_set_gen(Step *st, const GenArgs &g, cudaStream_t s, int nseq, const unsigned long long *seeds) {
    launch_k(k_set_gen, nseq, 1, 0, s, st, g, seeds);
}
void launch_stamp(Step *st, int idx, cudaStream_t s) { launch_k(k_stamp, 1, 1, 0, s, st, idx); }
void launch_conf(const float *logits, int ld, int nv, const Step *ms, Step *st, cudaStream_t s) {
    launch_k(k_conf, 1, 1024, 0, s, logits, ld, nv, ms, st);
}
void launch_set_pass_seqs(Step *st, const SeqPass *dev_passes, int nseq, cudaStream_t s) {
    launch_k(k_set_pass_seqs, nseq, 32, 0, s, st, dev_passes);
}
void launch_count_done(const Step *st, int nseq, int *ndone, cudaStream_t s) {
    launch_k(k_count_done, 1, 256, 0, s, st, nseq, ndone);
}
int kernels_init(int max_ctx, int hd, int rep) {
    // the largest carveout for the kernels of a verify round that take no dynamic shared memory
    max_carveout(k_embed);
    max_carveout(k_attn_prep);
    max_carveout(k_argmax_final);
    max_carveout(k_argmax_keys);
    max_carveout(k_keys_argmax);
    max_carveout(k_pass_end);
    max_carveout(k_accept);
    max_carveout(k_norm_rows);
    max_carveout(k_norm_quant);
    max_carveout(k_deltanet3<4, 4, PINFER_SPEC_MAX_K>);
    max_carveout(k_deltanet3<4, kMaxRows, PINFER_SPEC_MAX_K>);
    max_carveout(k_deltanet_prep<4>);
    max_carveout(k_deltanet_post);
    raise_smem(k_deltanet_rows, sizeof(float) * 2 * kDnBlk * kDnRec);
    // raise the dynamic shared memory limits once, outside any stream capture
    raise_smem(k_matvec<1, 0>, mv_smem<1>());
    raise_smem(k_matvec<1, 1>, mv_smem<1>());
    raise_smem(k_matvec<4, 0>, mv_smem<4>());
    raise_smem(k_matvec<4, 1>, mv_smem<4>());
    raise_smem(k_matvec<8, 0>, mv_smem<8>());
    raise_smem(k_matvec<8, 1>, mv_smem<8>());
    raise_smem(k_matvec<16, 0>, mv_smem<16>());
    raise_smem(k_matvec<16, 1>, mv_smem<16>());
    raise_smem(k_matvec_swiglu<1>, mv_smem<1>());
    raise_smem(k_matvec_swiglu<4>, mv_smem<4>());
    raise_smem(k_matvec_swiglu<8>, mv_smem<8>());
    raise_smem(k_matvec_swiglu<16>, mv_smem<16>());
    raise_smem(k_matvec_head<1>, mv_smem<1>());
    raise_smem(k_matvec_head<4>, mv_smem<4>());
    raise_smem(k_matvec_head<8>, mv_smem<8>());
    raise_smem(k_matvec_head<16>, mv_smem<16>());
    raise_smem(k_mv_head<1, false>);
    raise_smem(k_mv_head<1, true>);
    raise_smem(k_mv_head<4, false>);
    raise_smem(k_mv_head<4, true>);
    raise_smem(k_mv_head<8, false>);
    raise_smem(k_mv_head<8, true>);
    raise_smem(k_mv_head<16, false>);
    raise_smem(k_mv_head<16, true>);
    raise_smem(k_mv_head_mma<false>);
    raise_smem(k_mv_head_mma<true>);
    raise_smem(k_mv_panel<1, 0, false>);
    raise_smem(k_mv_panel<1, 1, false>);
    raise_smem(k_mv_panel<1, 3, false>);
    raise_smem(k_mv_panel<1, 0, true>);
    raise_smem(k_mv_panel<1, 3, true>);
    raise_smem(k_mv_panel<4, 0, false>);
    raise_smem(k_mv_panel<4, 1, false>);
    raise_smem(k_mv_panel<4, 3, false>);
    raise_smem(k_mv_panel<4, 0, true>);
    raise_smem(k_mv_panel<4, 3, true>);
    raise_smem(k_mv_panel<4, 0, true, 2>);
    raise_smem(k_mv_slice<0>);
    raise_smem(k_mv_slice<1>);
    if (max_ctx > 0) {
        raise_smem(k_deltanet2<4>, sizeof(float) * kDK * kDV);
        raise_smem(k_deltanet2<4, kMaxRows, PINFER_SPEC_MAX_K>, sizeof(float) * kDK * kDV);
        raise_smem(k_deltanet2<4, 4, 3>, sizeof(float) * kDK * kDV);
        raise_smem(k_deltanet, deltanet_smem(rep));
        raise_smem(k_attn, ((size_t)hd + max_ctx) * sizeof(float));
        raise_smem(k_attn2, attn2_smem(max_ctx));
        raise_smem(k_attn3, attn3_smem(max_ctx));
        raise_smem(k_attn4, attn4_smem(max_ctx));
        raise_smem(k_attn5<>, attn5_smem(max_ctx));
        raise_smem(k_attn5<4>, attn5_smem<4>(max_ctx));
        raise_smem(k_attn5<8>, attn5_smem<8>(max_ctx));
    }
    if (gemm_init() != 0) return -1;
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace nb
