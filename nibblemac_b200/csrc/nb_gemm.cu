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
// FMA chain runs on the CUDA cores, one thread per weight row, reading the dots back with
// tcgen05.ld. The chain, not the MMA, bounds the kernel.
//
// One CTA computes a tile of 128 weight rows (4 panels) x 64 activation rows over all columns:
//   warp 8       producer: per superblock (256 columns) the four 4608-byte weight units by bulk
//                copy, the A8 codes (two 128-column boxes, 128-byte swizzle) and the block
//                scales d / fsum by TMA tensor copies; then unpacks the 4-bit codes into int8 in
//                the tensor cores' K-major swizzled layout and pairs (d, fsum) per block.
//   warp 9       TMEM owner and MMA issuer: 8 MMAs (M 128, N 64, K 32) per superblock into a
//                ring of 8 TMEM slots of 64 columns, each completion signalled by tcgen05.commit.
//   warps 0..7   the chains: warp w reads TMEM lanes 32 (w % 4) .. (its 32 weight rows) and
//                activation rows 32 (w / 4) .. of the tile, and frees a slot as soon as its dots
//                are in registers.
// Two shared-memory stages; every wait is bounded (a timeout sets the status word, drains the
// copies and MMAs in flight, frees TMEM and returns).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "nb_dev.cuh"
#include "nb_engine.h"

namespace nb {

namespace {

constexpr int kGmM = 128;            // weight rows per tile (4 panels = TMEM lanes)
constexpr int kGmN = 64;             // activation rows per tile
constexpr int kGmSlots = 8;          // TMEM ring: one slot of kGmN columns per block
constexpr int kGmEpiWarps = 8;
constexpr int kGmProducer = kGmEpiWarps, kGmMma = kGmEpiWarps + 1;
constexpr int kGmThreads = (kGmEpiWarps + 2) * 32;
constexpr uint32_t kGmTmemCols = kGmSlots * kGmN;   // 512: the whole TMEM of the SM

// shared memory, from a 1024-byte aligned base (the swizzled operand tiles need it)
constexpr uint32_t kGmAStage = 2 * kGmM * 128;                 // unpacked codes [2 halves][128][128 B]
constexpr uint32_t kGmBStage = 2 * kGmN * 128;                 // A8 codes [2 halves][64][128 B]
constexpr uint32_t kGmRawStage = 4 * kUnitBytes;               // 4 weight units
constexpr uint32_t kGmQStage = kGmN * 8 * 4;                   // d or fsum [64][8] fp32
constexpr uint32_t kGmDfStage = 8 * kGmN * 2 * 4;              // (d, fsum) [8][64] pairs
constexpr uint32_t kGmA = 0;
constexpr uint32_t kGmB = kGmA + 2 * kGmAStage;
constexpr uint32_t kGmRaw = kGmB + 2 * kGmBStage;
constexpr uint32_t kGmDq = kGmRaw + 2 * kGmRawStage;
constexpr uint32_t kGmFq = kGmDq + 2 * kGmQStage;
constexpr uint32_t kGmDf = kGmFq + 2 * kGmQStage;
constexpr uint32_t kGmX = kGmDf + 2 * kGmDfStage;              // SwiGLU hand-off [2][2][32][32] fp32
constexpr uint32_t kGmBar = kGmX + 2 * 2 * 32 * 32 * 4;
constexpr uint32_t kGmMisc = kGmBar + 32 * 8;
constexpr uint32_t kGmSmem = kGmMisc + 64 + 1024;              // + alignment slack
static_assert(kGmSmem <= 227 * 1024, "shared memory of one CTA");
static_assert(kGmB % 1024 == 0 && kGmBStage % 1024 == 0 && kGmAStage % 1024 == 0, "swizzle atoms");

// instruction descriptor of tcgen05.mma kind::i8: D s32 (bits 4-5 = 2), A and B s8 (bits 7-9,
// 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t kGmIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGmN >> 3) << 17) |
                              ((uint32_t)(kGmM >> 4) << 24);

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
__device__ __forceinline__ void tm_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                 "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// a bounded wait whose outcome every lane of the (converged) warp agrees on, so the warp stays
// converged for the .sync.aligned tcgen05 instructions that follow
__device__ __forceinline__ bool wait_all(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}
__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// EPI 0: y[v][row] = acc; 1: y[v][row] += acc; 3: SwiGLU of (W0 = gate, W1 = up) and A8 of the
// product into `out`; 4: LM head, logits into y (may be null) and per-panel argmax keys.
template <int EPI>
__global__ void __launch_bounds__(kGmThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap td,
           const __grid_constant__ CUtensorMap tf, GemmArgs g) {
    extern __shared__ uint8_t gsm_raw[];
    const uint32_t raw_u = smem_u32(gsm_raw);
    const uint32_t sbase = (raw_u + 1023u) & ~1023u;
    uint8_t *sm = gsm_raw + (sbase - raw_u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kGmBar);
    uint64_t *full = bars, *unp = bars + 2, *sfree = bars + 4, *estage = bars + 6;
    uint64_t *mdone = bars + 8, *edone = bars + 16, *drain = bars + 24;
    uint32_t *tmem_at = reinterpret_cast<uint32_t *>(sm + kGmMisc);
    volatile int *abort_f = reinterpret_cast<volatile int *>(sm + kGmMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = g.n;
    const int ntn = (n + kGmN - 1) / kGmN;
    const int mt = blockIdx.x / ntn, n0 = (blockIdx.x % ntn) * kGmN;
    const int nsb = g.W0.nsb, nb = nsb * 8;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&unp[i], 32);
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
    if (warp == kGmMma) tm_alloc(tmem_at, kGmTmemCols);
    tm_fence_before();
    __syncthreads();
    tm_fence_after();
    const uint32_t tmem = *tmem_at;
    pdl_wait();
    pdl_trigger();

    if (warp == kGmProducer) {
        // unit u of the tile: EPI 3 interleaves gate and up panels (quarters 0 / 2 gate, 1 / 3 up)
        const uint8_t *ubase[4];
        bool uok[4];
        uint32_t wbytes = 0;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const Mat &m = (EPI == 3 && (u & 1)) ? g.W1 : g.W0;
            const int panel = EPI == 3 ? 2 * mt + (u >> 1) : 4 * mt + u;
            uok[u] = panel < m.npanels;
            ubase[u] = m.w + (size_t)panel * m.nsb * kUnitBytes;
            wbytes += uok[u] ? kUnitBytes : 0;
        }
        for (int s = 0; s < nsb; s++) {
            const int slot = s & 1;
            if (s >= 2) {
                const uint32_t par = (uint32_t)((s >> 1) - 1) & 1u;
                if (!wait_all(&sfree[slot], par) || !wait_all(&estage[slot], par)) {
                    *abort_f = 1;
                    break;
                }
            }
            uint8_t *rawp = sm + kGmRaw + slot * kGmRawStage;
            if (lane == 0) {
                mbar_arrive_expect(&full[slot], wbytes + kGmBStage + 2 * kGmQStage);
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (uok[u]) bulk_g2s(rawp + u * kUnitBytes, ubase[u] + (size_t)s * kUnitBytes, kUnitBytes, &full[slot]);
                uint8_t *bp = sm + kGmB + slot * kGmBStage;
                tma_load_2d(bp, &tq, s * 256, n0, &full[slot]);
                tma_load_2d(bp + kGmN * 128, &tq, s * 256 + 128, n0, &full[slot]);
                tma_load_2d(sm + kGmDq + slot * kGmQStage, &td, s * 8, n0, &full[slot]);
                tma_load_2d(sm + kGmFq + slot * kGmQStage, &tf, s * 8, n0, &full[slot]);
            }
            __syncwarp();
            if (!wait_all(&full[slot], (uint32_t)(s >> 1) & 1u)) {
                *abort_f = 1;
                wait_all(&full[slot], (uint32_t)(s >> 1) & 1u);   // the copies in flight, once more
                break;
            }
            // 4-bit codes -> int8, K-major with the 128-byte swizzle: row r of the tile, 16-byte
            // chunk j of a 128-column half at (r / 8) * 1024 + (r % 8) * 128 + ((j ^ r % 8) * 16);
            // block k's low nibbles are chunk 2 (k % 4), its high nibbles chunk 2 (k % 4) + 1
            uint8_t *ap = sm + kGmA + slot * kGmAStage;
            for (int idx = lane; idx < 4 * 8 * 32; idx += 32) {
                const int u = idx >> 8, k = (idx >> 5) & 7, r = idx & 31;
                const uint4 c = lds128(rawp + u * kUnitBytes + 512 * (k + 1) + r * 16);
                const uint4 lo = make_uint4(c.x & 0x0f0f0f0fu, c.y & 0x0f0f0f0fu, c.z & 0x0f0f0f0fu, c.w & 0x0f0f0f0fu);
                const uint4 hi = make_uint4((c.x >> 4) & 0x0f0f0f0fu, (c.y >> 4) & 0x0f0f0f0fu,
                                            (c.z >> 4) & 0x0f0f0f0fu, (c.w >> 4) & 0x0f0f0f0fu);
                const int row = u * 32 + r, rr = row & 7, j0 = (k & 3) * 2;
                uint8_t *rowp = ap + (k >> 2) * (kGmM * 128) + (row >> 3) * 1024 + rr * 128;
                *reinterpret_cast<uint4 *>(rowp + ((j0 ^ rr) << 4)) = lo;
                *reinterpret_cast<uint4 *>(rowp + (((j0 + 1) ^ rr) << 4)) = hi;
            }
            // (d, fsum) of activation row t and block k side by side: df[k][t]
            const float *dq = reinterpret_cast<const float *>(sm + kGmDq + slot * kGmQStage);
            const float *fq = reinterpret_cast<const float *>(sm + kGmFq + slot * kGmQStage);
            float2 *df = reinterpret_cast<float2 *>(sm + kGmDf + slot * kGmDfStage);
            for (int idx = lane; idx < 8 * kGmN; idx += 32) {
                const int k = idx / kGmN, t = idx % kGmN;
                df[idx] = make_float2(dq[t * 8 + k], fq[t * 8 + k]);
            }
            fence_proxy_async();   // the unpacked codes are read by the tensor cores
            mbar_arrive(&unp[slot]);
        }
    } else if (warp == kGmMma) {
        for (int b = 0; b < nb; b++) {
            const int s = b >> 3, k = b & 7, slot = s & 1, ts = b & (kGmSlots - 1);
            if (k == 0 && (!wait_all(&unp[slot], (uint32_t)(s >> 1) & 1u) ||
                           !wait_all(&full[slot], (uint32_t)(s >> 1) & 1u))) {
                *abort_f = 1;
                break;
            }
            if (b >= kGmSlots && !wait_all(&edone[ts], (uint32_t)((b >> 3) - 1) & 1u)) {
                *abort_f = 1;
                break;
            }
            tm_fence_after();
            if (lane == 0) {
                const uint32_t a = sbase + kGmA + slot * kGmAStage + (k >> 2) * (kGmM * 128) + (k & 3) * 32;
                const uint32_t bb = sbase + kGmB + slot * kGmBStage + (k >> 2) * (kGmN * 128) + (k & 3) * 32;
                tm_mma_i8(tmem + ts * kGmN, sw128_desc(a), sw128_desc(bb), kGmIdesc, 0u);
                tm_commit(&mdone[ts]);
                if (k == 7) tm_commit(&sfree[slot]);
            }
            __syncwarp();
        }
        if (lane == 0) tm_commit(drain);   // every MMA complete before TMEM is released
        __syncwarp();
        wait_all(drain, 0);
    } else {
        const int q = warp & 3, wg = warp >> 2;
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; i++) acc[i] = 0.0f;
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(wg * 32);
        for (int s = 0; s < nsb; s++) {
            const int slot = s & 1;
            if (__any_sync(0xffffffffu, *abort_f)) break;
            if (!wait_all(&unp[slot], (uint32_t)(s >> 1) & 1u)) {
                *abort_f = 1;
                break;
            }
            const uint4 sc = lds128(sm + kGmRaw + slot * kGmRawStage + q * kUnitBytes + lane * 16);
            const unsigned long long A = (unsigned long long)sc.x | ((unsigned long long)sc.y << 32);
            const unsigned long long B = (unsigned long long)sc.z | ((unsigned long long)sc.w << 32);
            const float D = half_bits_to_float((uint32_t)(A >> 48));
            const float M = half_bits_to_float((uint32_t)(B >> 48));
            const float4 *dfw = reinterpret_cast<const float4 *>(sm + kGmDf + slot * kGmDfStage) + wg * 16;
            bool ok = true;
#pragma unroll 1
            for (int k = 0; k < 8; k++) {
                const int b = s * 8 + k;
                const float ds = __fmul_rn(D, (float)(uint32_t)((A >> (6 * k)) & 63u));
                const float os = __fmul_rn(M, (float)(uint32_t)((B >> (6 * k)) & 63u));
                if (!wait_all(&mdone[k], (uint32_t)(b >> 3) & 1u)) {
                    ok = false;
                    break;
                }
                tm_fence_after();
                uint32_t is[32];
                tm_ld32(trow + (uint32_t)(k * kGmN), is);
                tm_wait_ld();
                tm_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&edone[k]);
                const float4 *dk = dfw + k * (kGmN / 2);
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float4 p = dk[i >> 1];   // d, fsum of rows i and i + 1
                    acc[i] = __fmaf_rn(__int2float_rn((int)is[i]), __fmul_rn(ds, p.x), acc[i]);
                    acc[i] = __fmaf_rn(-os, p.y, acc[i]);
                    acc[i + 1] = __fmaf_rn(__int2float_rn((int)is[i + 1]), __fmul_rn(ds, p.z), acc[i + 1]);
                    acc[i + 1] = __fmaf_rn(-os, p.w, acc[i + 1]);
                }
            }
            if (!ok) {
                *abort_f = 1;
                break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&estage[slot]);
        }
        const int vb = n0 + wg * 32;
        // one read of the flag per warp: both warps of a SwiGLU pair pass the named barrier below
        // whatever they read
        const bool live = !__any_sync(0xffffffffu, *abort_f);
        if (EPI == 3) {
            float *xch = reinterpret_cast<float *>(sm + kGmX) + ((q >> 1) * 2 + wg) * 32 * 32;
            if ((q & 1) && live) {
#pragma unroll
                for (int i = 0; i < 32; i++) xch[i * 32 + lane] = acc[i];
            }
            named_bar(1 + (q >> 1) * 2 + wg, 64);
        }
        if (live) {
            if (EPI == 0 || EPI == 1) {
                const int row = mt * kGmM + q * 32 + lane;
                if (row < g.W0.rows) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        if (vb + i < n) {
                            float *p = g.y + (size_t)(vb + i) * g.ldy + row;
                            *p = EPI == 0 ? acc[i] : __fadd_rn(*p, acc[i]);
                        }
                    }
                }
            } else if (EPI == 4) {
                const int row = mt * kGmM + q * 32 + lane, panel = mt * 4 + q;
                const bool valid = row < g.W0.rows;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int v = vb + i;
                    if (v < n) {
                        if (g.y && valid) g.y[(size_t)v * g.ldy + row] = acc[i];
                        unsigned long long key = valid ? argmax_key(acc[i], g.row_base + row) : 0ull;
                        key = warp_max_u64(key);
                        if (lane == 0 && panel < g.W0.npanels) g.partial[(size_t)v * g.W0.npanels + panel] = key;
                        if (row == 0 && g.row_base == 0) g.nan0[v] = acc[i] != acc[i];
                    }
                }
            } else if (EPI == 3) {
                float *xch = reinterpret_cast<float *>(sm + kGmX) + ((q >> 1) * 2 + wg) * 32 * 32;
                const int panel = 2 * mt + (q >> 1);
                if (!(q & 1) && panel < g.W0.npanels) {
                    // h = silu(gate) * up in place, then A8 of each activation row's block
#pragma unroll
                    for (int i = 0; i < 32; i++) xch[i * 32 + lane] = __fmul_rn(pf_silu(acc[i]), xch[i * 32 + lane]);
                    __syncwarp();
                    const int nbo = g.out.cols >> 5;
#pragma unroll 1
                    for (int i = 0; i < 32; i++) {
                        const int v = vb + i;
                        if (v >= n) break;
                        quant_block_warp(xch[i * 32 + lane], lane, g.out.q + (size_t)v * g.out.cols + panel * 32,
                                         g.out.d + (size_t)v * nbo + panel, g.out.fs + (size_t)v * nbo + panel);
                    }
                }
            }
        }
    }
    tm_fence_before();
    __syncthreads();
    if (warp == kGmMma) {
        tm_fence_after();
        tm_dealloc(tmem, kGmTmemCols);
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

template <int EPI>
void gemm_t(const GemmMaps &maps, const GemmArgs &g, cudaStream_t s) {
    const int ntn = (g.n + kGmN - 1) / kGmN;
    const int mtiles = EPI == 3 ? (g.W0.npanels + 1) / 2 : (g.W0.npanels + 3) / 4;
    launch_k(k_gemm<EPI>, dim3((unsigned)(mtiles * ntn)), dim3(kGmThreads), (size_t)kGmSmem, s,
             maps.q, maps.d, maps.fs, g);
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
    cuuint32_t qbox[2] = {128, (cuuint32_t)kGmN};
    cuuint64_t ddim[2] = {(cuuint64_t)nb, (cuuint64_t)nrows};
    cuuint64_t dstr[1] = {(cuuint64_t)nb * 4};
    cuuint32_t dbox[2] = {8, (cuuint32_t)kGmN};
    cuuint32_t one[2] = {1, 1};
    CUresult r0 = enc(&m->q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.q, qdim, qstr, qbox, one,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r1 = enc(&m->d, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.d, ddim, dstr, dbox, one,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = enc(&m->fs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.fs, ddim, dstr, dbox, one,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r0 != CUDA_SUCCESS || r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS) {
        char b[160];
        snprintf(b, sizeof b, "cuTensorMapEncodeTiled failed (%d %d %d)", (int)r0, (int)r1, (int)r2);
        set_last_error(b);
        return -1;
    }
    m->rows = nrows;
    m->cols = a.cols;
    return 0;
}

int gemm_init() {
    const int s = (int)kGmSmem;
    if (cudaFuncSetAttribute(k_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, s) != cudaSuccess)
        return -1;
    return 0;
}

void launch_gemm(int epi, const GemmMaps &maps, const GemmArgs &g, cudaStream_t s) {
    switch (epi) {
        case 0: gemm_t<0>(maps, g, s); break;
        case 1: gemm_t<1>(maps, g, s); break;
        case 3: gemm_t<3>(maps, g, s); break;
        default: gemm_t<4>(maps, g, s); break;
    }
}

}  // namespace nb
