// Q4K x A8 GEMM on the fifth-generation tensor cores (tcgen05, sm_100a), for passes of 17 and
// more activation rows: batched prefill and the multi-sequence verify batch.
//
// The result is bit-identical to the matvec kernels and to the reference (kern_q4k / q4_tile /
// q4_block, engine/src/kern_quant.c:148-245): per (weight row r, activation row v) and per
// 32-column block b in column order
//   isum = sum_j u[r][j] * q[v][j]                       (int32, exact)
//   acc  = fmaf((float)isum, (D_r * s6[b][r]) * d[b][v], acc)
//   acc  = fmaf(-(M_r * m6[b][r]), fsum[b][v], acc)
// The tensor cores compute the block dots only: one tcgen05.mma of kind::i8 with K = 32 is
// exactly one block, so every block's int32 dots land in their own TMEM columns, and the ordered
// FMA chain runs on the CUDA cores, one thread per (weight row, activation row pair), reading
// the dots back with tcgen05.ld. The chain, not the MMA, bounds the kernel.
//
// Weights: at 17+ rows the pass is compute-bound, so the tensor-core path reads a second copy
// of each matrix made once at load, the "tile image": per tile of 128 rows (4 panels) and
// superblock (256 columns) 34,816 bytes = the 4-bit codes widened to int8 in the tensor cores'
// K-major 128-byte-swizzled layout (32 KB, exactly the shared-memory image the MMA reads) and
// the 4 panels' scale entries (2 KB). One bulk copy per stage brings it in; nothing is unpacked
// on the hot path. (The CUDA-core matvec kernels keep reading the packed panels.)
//
// Persistent CTAs, one per SM, walk tiles of 128 weight rows x N activation rows (activation
// tiles fastest, so concurrent CTAs share weight tiles in L2). N is 64, or 32 / 16 when a pass
// has too few tiles of 64 rows to occupy half the SMs (a 64-row prefill chunk through a 1024-row
// projection has 8): each CTA then runs a quarter of the chains, which bound it.
//   warp 16      producer: per stage (one superblock of one tile) the tile-image chunk by bulk
//                copy, the A8 codes (two 128-column boxes, 128-byte swizzle) and the block
//                scales d / fsum by TMA tensor copies, into a ring of 3 stages.
//   warp 17      TMEM owner and MMA issuer: pairs (d, fsum) per block for the chains, then 8 MMAs
//                (M 128, N, K 32) per stage into a ring of 8 TMEM slots of N columns, each
//                completion signalled by tcgen05.commit.
//   warps 0..15  the chains: warp w reads TMEM lanes 32 (w % 4) .. (its 32 weight rows) and
//                activation rows (N / 4) (w / 4) .. of the tile, frees a TMEM slot as soon as its
//                dots are in registers, and writes the tile's outputs after the last stage.
// Every wait is bounded: a timeout sets the status word, lets the copies and MMAs in flight
// finish, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "nb_dev.cuh"
#include "nb_engine.h"

namespace nb {

namespace {

constexpr int kGmM = 128;            // weight rows per tile (4 panels = TMEM lanes)
constexpr int kGmSlots = 8;          // TMEM ring: one slot of N columns per block
constexpr int kGmStages = 3;         // shared-memory ring
constexpr int kGmEpiWarps = 16;      // 4 warpgroups; warpgroup g takes activation rows g N / 4 ..
constexpr int kGmWg = kGmEpiWarps / 4;
constexpr int kGmProducer = kGmEpiWarps, kGmMma = kGmEpiWarps + 1;
constexpr int kGmThreads = (kGmEpiWarps + 2) * 32;
constexpr uint32_t kGmACodes = 2 * kGmM * 128;                 // int8 codes [2 halves][128 rows][128 B]
constexpr uint32_t kGmTileBytes = kGmACodes + 4 * 512;         // + 4 panels' scale entries

// The activation tile height N (16, 32 or 64 rows) sets everything else: a pass with few weight
// tiles takes a smaller N so that more CTAs share the work (the FMA chains, one per weight row
// and activation row, are what bounds a CTA).
template <int N>
struct GmCfg {
    static_assert(N == 16 || N == 32 || N == 64, "activation tile height");
    static constexpr int kTpt = N / kGmWg;                            // activation rows per epilogue thread
    static constexpr uint32_t kTmemCols = kGmSlots * N;              // a power of two >= 32
    // one stage of shared memory (1024-byte aligned: the swizzled operand tiles need it)
    static constexpr uint32_t kBStage = 2 * N * 128;                 // A8 codes [2 halves][N rows][128 B]
    static constexpr uint32_t kQStage = N * 8 * 4;                   // d or fsum [N rows][8 blocks] fp32
    static constexpr uint32_t kDfStage = 8 * N * 2 * 4;              // [8 blocks][N / 2] (d_t, d_t+1, fs_t, fs_t+1)
    static constexpr uint32_t kOffB = kGmTileBytes;
    static constexpr uint32_t kOffDq = kOffB + kBStage;
    static constexpr uint32_t kOffFq = kOffDq + kQStage;
    static constexpr uint32_t kOffDf = kOffFq + kQStage;
    static constexpr uint32_t kStageBytes = kOffDf + kDfStage;
    static constexpr uint32_t kBar = kGmStages * kStageBytes;
    static constexpr uint32_t kMisc = kBar + 32 * 8;
    static constexpr uint32_t kSmem = kMisc + 64 + 1024;              // + alignment slack
    static_assert(kSmem <= 227 * 1024, "shared memory of one CTA");
    static_assert(kStageBytes % 1024 == 0 && kOffB % 1024 == 0 && kGmACodes % 2048 == 0, "swizzle atoms");
    // instruction descriptor of tcgen05.mma kind::i8: D s32 (bits 4-5 = 2), A and B s8 (bits 7-9,
    // 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
    static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                                       ((uint32_t)(kGmM >> 4) << 24);
};
constexpr int gm_index(int N) { return N == 16 ? 0 : N == 32 ? 1 : 2; }

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart
// (start >> 4 in bits 0-13, leading offset 16 B, stride offset 1024 B at bit 32, version 1 at
// bit 46, layout type 2 = SWIZZLE_128B at bit 61)
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 2-D TMA tensor copy global -> shared completing on `bar` (x = innermost coordinate)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tm_alloc(uint32_t *dst, uint32_t ncols) {   // one full warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tm_dealloc(uint32_t taddr, uint32_t ncols) {   // the same warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] = A B (accumulate = 0) or += (accumulate = 1); issued by one thread
__device__ __forceinline__ void tm_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void tm_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 consecutive columns of this thread's TMEM lane
[[maybe_unused]] __device__ __forceinline__ void tm_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                 "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tm_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tm_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tm_ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void tm_ld(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) tm_ld32(taddr, r);
    else if constexpr (N == 16) tm_ld16(taddr, r);
    else if constexpr (N == 8) tm_ld8(taddr, r);
    else tm_ld4(taddr, r);
}
// (float)v for |v| < 2^22, exactly, without the conversion unit: the bits of 1.5 * 2^23 + v
// read as a float are 12582912 + v, and subtracting 12582912 is exact
__device__ __forceinline__ float int_bits_plus_magic(uint32_t v) { return __int_as_float((int)v + 0x4B400000); }
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// a bounded wait whose outcome every lane of the (converged) warp agrees on, so the warp stays
// converged for the .sync.aligned tcgen05 instructions that follow
__device__ __forceinline__ bool wait_all(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Widen one tile image chunk per CTA (blockIdx.x = tile, blockIdx.y = superblock): tile t holds
// panels 4t .. 4t + 3 of the row concatenation W0 ++ W1 (W1.npanels may be 0); rows past the
// end are zero. Row r of the tile, 16-byte chunk j of a 128-column half lands at
// (r / 8) * 1024 + (r % 8) * 128 + ((j ^ r % 8) * 16); block k's low nibbles (columns 0..15)
// are chunk 2 (k % 4) of half k / 4, its high nibbles (columns 16..31) chunk 2 (k % 4) + 1.
__global__ void k_gemm_tile(Mat W0, Mat W1, uint8_t *dst) {
    const int mt = blockIdx.x, sb = blockIdx.y;
    uint8_t *o = dst + ((size_t)mt * W0.nsb + sb) * kGmTileBytes;
    for (int idx = threadIdx.x; idx < 4 * 9 * 32; idx += blockDim.x) {
        const int u = idx / 288, k = (idx % 288) / 32 - 1, r = idx % 32;   // k = -1: the scale entry
        const int p = 4 * mt + u;
        const Mat *m = p < W0.npanels ? &W0 : (p - W0.npanels < W1.npanels ? &W1 : nullptr);
        const int pp = p < W0.npanels ? p : p - W0.npanels;
        uint4 c = make_uint4(0u, 0u, 0u, 0u);
        if (m) c = *reinterpret_cast<const uint4 *>(m->w + ((size_t)pp * m->nsb + sb) * kUnitBytes + (k + 1) * 512 + r * 16);
        if (k < 0) {
            *reinterpret_cast<uint4 *>(o + kGmACodes + u * 512 + r * 16) = c;
            continue;
        }
        const uint4 lo = make_uint4(c.x & 0x0f0f0f0fu, c.y & 0x0f0f0f0fu, c.z & 0x0f0f0f0fu, c.w & 0x0f0f0f0fu);
        const uint4 hi = make_uint4((c.x >> 4) & 0x0f0f0f0fu, (c.y >> 4) & 0x0f0f0f0fu, (c.z >> 4) & 0x0f0f0f0fu,
                                    (c.w >> 4) & 0x0f0f0f0fu);
        const int row = u * 32 + r, rr = row & 7, j0 = (k & 3) * 2;
        uint8_t *rowp = o + (k >> 2) * (kGmM * 128) + (row >> 3) * 1024 + rr * 128;
        *reinterpret_cast<uint4 *>(rowp + ((j0 ^ rr) << 4)) = lo;
        *reinterpret_cast<uint4 *>(rowp + (((j0 + 1) ^ rr) << 4)) = hi;
    }
}

// SwiGLU of a pass's gate / up rows and A8 of the product (pf_mlp / pf_silu_mul,
// engine/src/forward.c:49-58, then kern_quant_act): y [n][ldy] holds gate in columns [0, ffn)
// and up in [ffn, 2 ffn); one warp per (row, 32-column block).
__global__ void k_swiglu_quant(const float *y, int ldy, int ffn, int n, Act out) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nbo = ffn >> 5;
    if (gw >= (long long)n * nbo) return;
    const int v = (int)(gw / nbo), b = (int)(gw % nbo);
    const float *yr = y + (size_t)v * ldy + b * 32 + lane;
    const float h = __fmul_rn(pf_silu(yr[0]), yr[ffn]);
    quant_block_warp(h, lane, out.q + (size_t)v * out.cols + b * 32, out.d + (size_t)v * nbo + b,
                     out.fs + (size_t)v * nbo + b);
}

// EPI 0: y[v][row] = acc; 1: y[v][row] += acc (the residual stream); 4: LM head, logits into y
// (may be null) and per-panel argmax keys.
template <int EPI, int N>
__global__ void __launch_bounds__(kGmThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap td,
           const __grid_constant__ CUtensorMap tf, GemmArgs g) {
    using Cfg = GmCfg<N>;
    extern __shared__ uint8_t gsm_raw[];
    const uint32_t raw_u = smem_u32(gsm_raw);
    const uint32_t sbase = (raw_u + 1023u) & ~1023u;
    uint8_t *sm = gsm_raw + (sbase - raw_u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + Cfg::kBar);
    uint64_t *full = bars, *ready = bars + 3, *sfree = bars + 6, *estage = bars + 9;
    uint64_t *mdone = bars + 12, *edone = bars + 20, *drain = bars + 28;
    uint32_t *tmem_at = reinterpret_cast<uint32_t *>(sm + Cfg::kMisc);
    volatile int *abort_f = reinterpret_cast<volatile int *>(sm + Cfg::kMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = g.n, nsb = g.W.nsb;
    const int ntn = (n + N - 1) / N, ntiles = g.W.mtiles * ntn;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGmStages; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&ready[i], 32);
            mbar_init(&sfree[i], 1);
            mbar_init(&estage[i], kGmEpiWarps);
        }
        for (int i = 0; i < kGmSlots; i++) {
            mbar_init(&mdone[i], 1);
            mbar_init(&edone[i], kGmEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_f = 0;
        fence_mbar_init();
    }
    if (warp == kGmMma) tm_alloc(tmem_at, Cfg::kTmemCols);
    tm_fence_before();
    __syncthreads();
    tm_fence_after();
    const uint32_t tmem = *tmem_at;
    pdl_wait();
    pdl_trigger();

    if (warp == kGmProducer) {
        int gs = 0;   // stages issued by this CTA
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            const int mt = tile / ntn, n0 = (tile % ntn) * N;
            const uint8_t *wt = g.W.t + (size_t)mt * nsb * kGmTileBytes;
            for (int s = 0; s < nsb; s++, gs++) {
                const int slot = gs % kGmStages;
                const uint32_t use = (uint32_t)(gs / kGmStages);
                if (gs >= kGmStages && (!wait_all(&sfree[slot], (use - 1) & 1u) || !wait_all(&estage[slot], (use - 1) & 1u))) {
                    *abort_f = 1;
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    uint8_t *st = sm + slot * Cfg::kStageBytes;
                    mbar_arrive_expect(&full[slot], kGmTileBytes + Cfg::kBStage + 2 * Cfg::kQStage);
                    bulk_g2s(st, wt + (size_t)s * kGmTileBytes, kGmTileBytes, &full[slot]);
                    tma_load_2d(st + Cfg::kOffB, &tq, s * 256, n0, &full[slot]);
                    tma_load_2d(st + Cfg::kOffB + N * 128, &tq, s * 256 + 128, n0, &full[slot]);
                    tma_load_2d(st + Cfg::kOffDq, &td, s * 8, n0, &full[slot]);
                    tma_load_2d(st + Cfg::kOffFq, &tf, s * 8, n0, &full[slot]);
                }
                __syncwarp();
            }
        }
        // the last stages' copies have landed before shared memory is released (normally the
        // MMA warp already waited for them)
        for (int i = gs > kGmStages ? gs - kGmStages : 0; i < gs; i++)
            wait_all(&full[i % kGmStages], (uint32_t)(i / kGmStages) & 1u);
    } else if (warp == kGmMma) {
        int gs = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            for (int s = 0; s < nsb; s++, gs++) {
                const int slot = gs % kGmStages;
                const uint32_t use = (uint32_t)(gs / kGmStages);
                if (!wait_all(&full[slot], use & 1u)) {
                    *abort_f = 1;
                    ok = false;
                    break;
                }
                uint8_t *st = sm + slot * Cfg::kStageBytes;
                // (d_t, d_t+1, fsum_t, fsum_t+1) per block and activation-row pair for the chains
                const float *dq = reinterpret_cast<const float *>(st + Cfg::kOffDq);
                const float *fq = reinterpret_cast<const float *>(st + Cfg::kOffFq);
                float4 *df = reinterpret_cast<float4 *>(st + Cfg::kOffDf);
                for (int idx = lane; idx < 8 * N / 2; idx += 32) {
                    const int k = idx / (N / 2), t = (idx % (N / 2)) * 2;
                    df[idx] = make_float4(dq[t * 8 + k], dq[(t + 1) * 8 + k], fq[t * 8 + k], fq[(t + 1) * 8 + k]);
                }
                mbar_arrive(&ready[slot]);
                for (int k = 0; k < 8; k++) {
                    if (gs >= 1 && !wait_all(&edone[k], (uint32_t)(gs - 1) & 1u)) {
                        *abort_f = 1;
                        ok = false;
                        break;
                    }
                    tm_fence_after();
                    if (lane == 0) {
                        const uint32_t a = sbase + slot * Cfg::kStageBytes + (k >> 2) * (kGmM * 128) + (k & 3) * 32;
                        const uint32_t b = sbase + slot * Cfg::kStageBytes + Cfg::kOffB + (k >> 2) * (N * 128) + (k & 3) * 32;
                        tm_mma_i8(tmem + k * N, sw128_desc(a), sw128_desc(b), Cfg::kIdesc, 0u);
                        tm_commit(&mdone[k]);
                        if (k == 7) tm_commit(&sfree[slot]);
                    }
                    __syncwarp();
                }
                if (!ok) break;
            }
        }
        if (lane == 0) tm_commit(drain);   // every MMA complete before TMEM is released
        __syncwarp();
        wait_all(drain, 0);
    } else {
        const int q = warp & 3, wg = warp >> 2;
        const float2 magic = make_float2(-12582912.0f, -12582912.0f);
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(wg * Cfg::kTpt);
        int gs = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            const int mt = tile / ntn, n0 = (tile % ntn) * N;
            // two activation rows per packed f32x2 chain: acc[j] = rows (2 j, 2 j + 1) of this thread
            float2 acc[Cfg::kTpt / 2];
#pragma unroll
            for (int j = 0; j < Cfg::kTpt / 2; j++) acc[j] = make_float2(0.0f, 0.0f);
            for (int s = 0; s < nsb; s++, gs++) {
                const int slot = gs % kGmStages;
                if (__any_sync(0xffffffffu, *abort_f) || !wait_all(&ready[slot], (uint32_t)(gs / kGmStages) & 1u)) {
                    *abort_f = 1;
                    ok = false;
                    break;
                }
                const uint8_t *st = sm + slot * Cfg::kStageBytes;
                const uint4 sc = lds128(st + kGmACodes + q * 512 + lane * 16);
                const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
                const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
                const float D = half_bits_to_float((uint32_t)(A >> 48));
                const float M = half_bits_to_float((uint32_t)(B >> 48));
                const float4 *dfw = reinterpret_cast<const float4 *>(st + Cfg::kOffDf) + wg * (Cfg::kTpt / 2);
                // blocks in pairs: the commit after block k + 1's MMA also covers block k's
                // (tcgen05.commit tracks every earlier MMA of the issuing thread), so one wait,
                // one TMEM-load wait and one fence pair serve both
#pragma unroll 1
                for (int k = 0; k < 8; k += 2) {
                    if (!wait_all(&mdone[k + 1], (uint32_t)gs & 1u)) {
                        ok = false;
                        break;
                    }
                    tm_fence_after();
                    uint32_t is[2][Cfg::kTpt];
                    tm_ld(trow + (uint32_t)(k * N), is[0]);
                    tm_ld(trow + (uint32_t)((k + 1) * N), is[1]);
                    tm_wait_ld();
                    tm_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&edone[k]);
                        mbar_arrive(&edone[k + 1]);
                    }
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const int kb = k + kk;
                        const float ds = __fmul_rn(D, (float)(uint32_t)((A >> (6 * kb)) & 63u));
                        const float os = __fmul_rn(M, (float)(uint32_t)((B >> (6 * kb)) & 63u));
                        const float2 ds2 = make_float2(ds, ds), nos2 = make_float2(-os, -os);
                        const float4 *dk = dfw + kb * (N / 2);
                        // per row: acc = fmaf((float)isum, ds * d, acc); acc = fmaf(-os, fsum, acc),
                        // two rows per packed instruction (each lane of f32x2 rounds as the scalar op)
#pragma unroll
                        for (int j = 0; j < Cfg::kTpt / 2; j++) {
                            const float4 p = dk[j];   // d_2j, d_2j+1, fsum_2j, fsum_2j+1
                            const float2 f = __fadd2_rn(make_float2(int_bits_plus_magic(is[kk][2 * j]),
                                                                    int_bits_plus_magic(is[kk][2 * j + 1])), magic);
                            acc[j] = __ffma2_rn(f, __fmul2_rn(ds2, make_float2(p.x, p.y)), acc[j]);
                            acc[j] = __ffma2_rn(nos2, make_float2(p.z, p.w), acc[j]);
                        }
                    }
                }
                if (!ok) {
                    *abort_f = 1;
                    break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&estage[slot]);
            }
            if (!ok) break;
            // the tile's outputs (stores of consecutive weight rows by consecutive lanes)
            const int vb = n0 + wg * Cfg::kTpt, row = mt * kGmM + q * 32 + lane;
            const bool valid = row < g.W.rows;
#pragma unroll
            for (int i = 0; i < Cfg::kTpt; i++) {
                const int v = vb + i;
                const float a = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
                if (v < n) {
                    if (EPI == 0 || EPI == 1) {
                        if (valid) {
                            float *p = g.y + (size_t)v * g.ldy + row;
                            *p = EPI == 0 ? a : __fadd_rn(*p, a);
                        }
                    } else {
                        if (g.y && valid) g.y[(size_t)v * g.ldy + row] = a;
                        const unsigned long long key = warp_max_u64(valid ? argmax_key(a, g.row_base + row) : 0ull);
                        const int panel = mt * 4 + q;
                        if (lane == 0 && panel < g.W.npanels) g.partial[(size_t)v * g.W.npanels + panel] = key;
                        if (row == 0 && g.row_base == 0) g.nan0[v] = a != a;
                    }
                }
            }
        }
    }
    tm_fence_before();
    __syncthreads();
    if (warp == kGmMma) {
        tm_fence_after();
        tm_dealloc(tmem, Cfg::kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_f && g.status) *g.status = -91;   // a device wait timed out
}

// ---- host: TMA tensor maps over an A8 activation buffer
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int sm_count() {
    static int n = 0;
    static std::once_flag once;
    std::call_once(once, [] {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
    });
    return n;
}

template <int EPI, int N>
void gemm_n(const GemmMaps &maps, const GemmArgs &g, cudaStream_t s) {
    const int ntiles = g.W.mtiles * ((g.n + N - 1) / N);
    const int grid = ntiles < sm_count() ? ntiles : sm_count();
    const int i = gm_index(N);
    launch_k(k_gemm<EPI, N>, dim3((unsigned)grid), dim3(kGmThreads), (size_t)GmCfg<N>::kSmem, s, maps.q[i], maps.d[i],
             maps.fs[i], g);
}

// The tallest activation tile that still gives at least half the SMs a tile, else 16 rows.
template <int EPI>
void gemm_t(const GemmMaps &maps, const GemmArgs &g, cudaStream_t s) {
    const int half = sm_count() / 2;
    if (g.W.mtiles * ((g.n + 63) / 64) >= half) gemm_n<EPI, 64>(maps, g, s);
    else if (g.W.mtiles * ((g.n + 31) / 32) >= half) gemm_n<EPI, 32>(maps, g, s);
    else gemm_n<EPI, 16>(maps, g, s);
}

}  // namespace

int gemm_maps(const Act &a, int nrows, GemmMaps *m) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) {
        set_last_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
        return -1;
    }
    if (a.cols % 256 || nrows < 1 || ((uintptr_t)a.q & 15) || ((uintptr_t)a.d & 15) || ((uintptr_t)a.fs & 15)) {
        set_last_error("gemm_maps: A8 buffer not 16-byte aligned or columns not a multiple of 256");
        return -1;
    }
    const int nb = a.cols / 32;
    cuuint64_t qdim[2] = {(cuuint64_t)a.cols, (cuuint64_t)nrows};
    cuuint64_t qstr[1] = {(cuuint64_t)a.cols};
    cuuint64_t ddim[2] = {(cuuint64_t)nb, (cuuint64_t)nrows};
    cuuint64_t dstr[1] = {(cuuint64_t)nb * 4};
    cuuint32_t one[2] = {1, 1};
    for (int i = 0; i < 3; i++) {   // activation tile heights 16, 32, 64
        const cuuint32_t h = 16u << i;
        cuuint32_t qbox[2] = {128, h};
        cuuint32_t dbox[2] = {8, h};
        CUresult r0 = enc(&m->q[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.q, qdim, qstr, qbox, one,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        CUresult r1 = enc(&m->d[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.d, ddim, dstr, dbox, one,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        CUresult r2 = enc(&m->fs[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.fs, ddim, dstr, dbox, one,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r0 != CUDA_SUCCESS || r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS) {
            char b[160];
            snprintf(b, sizeof b, "cuTensorMapEncodeTiled failed (%d %d %d)", (int)r0, (int)r1, (int)r2);
            set_last_error(b);
            return -1;
        }
    }
    m->rows = nrows;
    m->cols = a.cols;
    return 0;
}

template <int N>
bool gemm_init_n() {
    const int s = (int)GmCfg<N>::kSmem;
    return cudaFuncSetAttribute(k_gemm<0, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) == cudaSuccess &&
           cudaFuncSetAttribute(k_gemm<1, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) == cudaSuccess &&
           cudaFuncSetAttribute(k_gemm<4, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) == cudaSuccess;
}

int gemm_init() { return gemm_init_n<16>() && gemm_init_n<32>() && gemm_init_n<64>() ? 0 : -1; }

size_t gemm_tiled_bytes(int rows, int cols) {
    const int npanels = (rows + kPanelRows - 1) / kPanelRows;
    return (size_t)((npanels + 3) / 4) * (cols / 256) * kGmTileBytes;
}

GemmW gemm_w(const Mat &W0, const Mat &W1, uint8_t *tiled) {
    GemmW w;
    w.t = tiled;
    w.npanels = W0.npanels + W1.npanels;
    w.rows = W1.npanels ? W0.npanels * kPanelRows + W1.rows : W0.rows;
    w.cols = W0.cols;
    w.nsb = W0.nsb;
    w.mtiles = (w.npanels + 3) / 4;
    return w;
}

void launch_gemm_tile(const Mat &W0, const Mat &W1, uint8_t *tiled, cudaStream_t s) {
    const int mtiles = (W0.npanels + W1.npanels + 3) / 4;
    launch_k(k_gemm_tile, dim3((unsigned)mtiles, (unsigned)W0.nsb), dim3(256), 0, s, W0, W1, tiled);
}

void launch_gemm(int epi, const GemmMaps &maps, const GemmArgs &g, cudaStream_t s) {
    switch (epi) {
        case 0: gemm_t<0>(maps, g, s); break;
        case 1: gemm_t<1>(maps, g, s); break;
        default: gemm_t<4>(maps, g, s); break;
    }
}

void launch_swiglu_quant(const float *y, int ldy, int ffn, int n, Act out, cudaStream_t s) {
    const long long warps = (long long)n * (ffn / 32);
    launch_k(k_swiglu_quant, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, s, y, ldy, ffn, n, out);
}

}  // namespace nb
