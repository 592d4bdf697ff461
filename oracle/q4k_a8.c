/* CPU oracle for the Q4K x A8 path: TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Scalar restatement of the reference's quantised-matvec arithmetic. Build flags:
 * -O2 -std=c11 -ffp-contract=off (the reference's HOST_CFLAGS, engine/Makefile:33). */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define SB_COLS 256
#define SB_BYTES 576
#define SCALE_BYTES 64

static float h2f(const uint8_t *p) {
    _Float16 h;
    memcpy(&h, p, 2);
    return (float)h;
}

/* kern_quant_act (engine/src/kern_act.c:14-41): per block of 32 columns amax = max |x|,
 * id = amax > 0 ? 127 / amax : 0, q = round-half-even(x * id) (vcvtnq), d = amax / 127,
 * fsum = d * (float)sum(q). Block-major: element (b, v) at index b * n + v. */
void or_quant_act(const float *X, int n, int cols, int8_t *q, float *d, float *fsum) {
    const int nb = cols / 32;
    for (int v = 0; v < n; v++)
        for (int b = 0; b < nb; b++) {
            const float *x = X + (size_t)v * cols + b * 32;
            float amax = 0.0f;
            for (int j = 0; j < 32; j++) {
                const float a = fabsf(x[j]);
                if (a > amax) amax = a;
            }
            const float id = amax > 0.0f ? 127.0f / amax : 0.0f;
            const size_t k = (size_t)b * n + v;
            int sum = 0;
            for (int j = 0; j < 32; j++) {
                const float y = rintf(x[j] * id);
                const int qi = y != y ? 0 : (int)y;   /* |y| <= 127 for finite x */
                q[k * 32 + j] = (int8_t)(qi > 127 ? 127 : qi < -128 ? -128 : qi);
                sum += qi;
            }
            d[k] = amax / 127.0f;
            fsum[k] = d[k] * (float)sum;
        }
}

/* kern_get6 (engine/src/kern_act.c:46-49): value j (0..31) of a 24-byte 6-bit array. */
static int get6(const uint8_t *p, int j) {
    const int lo = j < 16 ? p[j] & 15 : p[j - 16] >> 4;
    return lo | ((p[16 + j % 8] >> (2 * (j / 8))) & 3) << 4;
}

/* The per-(row, block) integer dot: sum over 32 columns of u4 code x int8 activation. Codes
 * of block k, row i sit at byte 64 + 64k + 16i of the superblock: byte j holds column j
 * (low nibble) and column j + 16 (high nibble) (engine/FORMAT.md "Nibbles"). */
static int32_t block_dot(const uint8_t *codes, const int8_t *x) {
    int32_t s = 0;
    for (int j = 0; j < 16; j++) {
        s += (int32_t)(codes[j] & 15) * x[j];
        s += (int32_t)(codes[j] >> 4) * x[j + 16];
    }
    return s;
}

void or_q4k_isums(const uint8_t *W, int rows, int cols, const int8_t *q, int n, int32_t *isum) {
    const int nsb = cols / SB_COLS, nb = cols / 32;
    for (int r = 0; r < rows; r++) {
        const uint8_t *tile = W + (size_t)(r / 4) * nsb * SB_BYTES;
        const int i = r % 4;
        for (int sb = 0; sb < nsb; sb++)
            for (int k = 0; k < 8; k++) {
                const uint8_t *codes = tile + (size_t)sb * SB_BYTES + SCALE_BYTES + k * 64 + i * 16;
                const int b = sb * 8 + k;
                for (int v = 0; v < n; v++)
                    isum[((size_t)v * rows + r) * nb + b] =
                        block_dot(codes, q + ((size_t)b * n + v) * 32);
            }
    }
}

/* kern_q4k -> q4_tile -> q4k_scales -> q4_block (engine/src/kern_quant.c:148-245,296-304),
 * per (row, vector), blocks in column order:
 *   ds = D * s6, os = M * m6 (both exact in fp32: 6-bit x 11-bit mantissa, :201-205)
 *   acc = fmaf((float)isum, ds * d_act, acc)      (vfmaq_f32 with vmulq_n_f32, :175)
 *   acc = fmaf(-os, fsum_act, acc)                (vfmsq_n_f32, :176)
 * The result does not depend on n or on the row split (:103-109). */
void or_q4k_matmul_act(const uint8_t *W, int rows, int cols, const int8_t *q, const float *d,
                       const float *fsum, int n, float *Y) {
    const int nsb = cols / SB_COLS;
    for (int r = 0; r < rows; r++) {
        const uint8_t *tile = W + (size_t)(r / 4) * nsb * SB_BYTES;
        const int i = r % 4;
        for (int v = 0; v < n; v++) {
            float acc = 0.0f;
            for (int sb = 0; sb < nsb; sb++) {
                const uint8_t *p = tile + (size_t)sb * SB_BYTES;
                const float D = h2f(p + 2 * i), M = h2f(p + 8 + 2 * i);
                for (int k = 0; k < 8; k++) {
                    const int b = sb * 8 + k;
                    const float ds = D * (float)get6(p + 16, 4 * k + i);
                    const float os = M * (float)get6(p + 40, 4 * k + i);
                    const size_t a = (size_t)b * n + v;
                    const int32_t s = block_dot(p + SCALE_BYTES + k * 64 + i * 16, q + a * 32);
                    acc = fmaf((float)s, ds * d[a], acc);
                    acc = fmaf(-os, fsum[a], acc);
                }
            }
            Y[(size_t)v * rows + r] = acc;
        }
    }
}

void or_q4k_matmul(const uint8_t *W, int rows, int cols, const float *X, int n, float *Y) {
    const int nb = cols / 32;
    int8_t *q = malloc((size_t)n * cols);
    float *d = malloc((size_t)n * nb * sizeof(float)), *fs = malloc((size_t)n * nb * sizeof(float));
    if (!q || !d || !fs) abort();
    or_quant_act(X, n, cols, q, d, fs);
    or_q4k_matmul_act(W, rows, cols, q, d, fs, n, Y);
    free(q);
    free(d);
    free(fs);
}

/* kern_get_row_q, Q4K branch (engine/src/kern_act.c:76-85): dd = D * s6, mm = M * m6,
 * value = dd * u - mm with two roundings (no fused multiply-add). */
void or_q4k_get_row(const uint8_t *W, int rows, int cols, int row, float *dst) {
    (void)rows;
    const int nsb = cols / SB_COLS, i = row % 4;
    const uint8_t *p = W + (size_t)(row / 4) * nsb * SB_BYTES;
    for (int sb = 0; sb < nsb; sb++, p += SB_BYTES, dst += SB_COLS) {
        const float D = h2f(p + 2 * i), M = h2f(p + 8 + 2 * i);
        for (int k = 0; k < 8; k++) {
            const float dd = D * (float)get6(p + 16, 4 * k + i);
            const float mm = M * (float)get6(p + 40, 4 * k + i);
            const uint8_t *c = p + SCALE_BYTES + k * 64 + i * 16;
            for (int j = 0; j < 16; j++) {
                dst[k * 32 + j] = dd * (float)(c[j] & 15) - mm;
                dst[k * 32 + 16 + j] = dd * (float)(c[j] >> 4) - mm;
            }
        }
    }
}

/* ---- kbench's seeded inputs (engine/bench/kbench_util.c) ----------------------------- */

/* xorshift64* (kbench_util.c:19-24) */
static uint64_t kb_next(uint64_t *s) {
    *s ^= *s >> 12;
    *s ^= *s << 25;
    *s ^= *s >> 27;
    return *s * 2685821657736338717ull;
}

/* sum of two 24-bit uniforms, centred, with every 64th value scaled by 6 (:27-35) */
static void kb_gen(float *w, size_t n, uint64_t *s, float scale) {
    for (size_t i = 0; i < n; i++) {
        const uint64_t r = kb_next(s);
        const float a = (float)(r >> 40) * (1.0f / 16777216.0f);
        const float b = (float)((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
        const float v = (a + b - 1.0f) * scale;
        w[i] = (r & 63) == 0 ? 6.0f * v : v;
    }
}

void or_kb_fill_vec(float *x, size_t n, uint64_t seed) {   /* :37-40 */
    uint64_t s = seed * 0x9E3779B97F4A7C15ull + 1;
    kb_gen(x, n, &s, 1.0f);
}

static float kb_clamp(float v, float lo, float hi) { return v < lo ? lo : v > hi ? hi : v; }

/* 6-bit packing as kern_get6 reads it (:100-107) */
static void kb_put6(uint8_t *p, const int *v) {
    memset(p, 0, 24);
    for (int j = 0; j < 32; j++) {
        p[j % 16] |= (uint8_t)((v[j] & 15) << (j < 16 ? 0 : 4));
        p[16 + j % 8] |= (uint8_t)((v[j] >> 4) << (2 * (j / 8)));
    }
}

/* kbench's benchmark-data Q4K packer (:109-138): per row min/max per group, fp16 D / M from
 * the row maxima, 6-bit scales rounded up so the 16 levels span the group, plain rounding of
 * the codes. (Not the converter's quantiser: benchmark data only.) */
static void kb_pack_q4k_sb(const float *w, int cols, uint8_t *p) {
    int s6[32], m6[32];
    for (int i = 0; i < 4; i++) {
        float dg[8], mg[8], dmax = 0, mmax = 0;
        for (int g = 0; g < 8; g++) {
            const float *x = w + (size_t)i * cols + g * 32;
            float mn = x[0], mx = x[0];
            for (int j = 1; j < 32; j++) mn = fminf(mn, x[j]), mx = fmaxf(mx, x[j]);
            mn = fminf(mn, 0.0f);
            dg[g] = (mx - mn) / 15.0f, mg[g] = -mn;
            dmax = fmaxf(dmax, dg[g]), mmax = fmaxf(mmax, mg[g]);
        }
        const _Float16 hd = (_Float16)(dmax / 63.0f), hm = (_Float16)(mmax / 63.0f);
        memcpy(p + 2 * i, &hd, 2);
        memcpy(p + 8 + 2 * i, &hm, 2);
        const float D = (float)hd, M = (float)hm;
        for (int g = 0; g < 8; g++) {
            s6[g * 4 + i] = D > 0 ? (int)fminf(ceilf(dg[g] / D), 63) : 0;
            m6[g * 4 + i] = M > 0 ? (int)lrintf(fminf(mg[g] / M, 63)) : 0;
            const float d = D * s6[g * 4 + i], m = M * m6[g * 4 + i], id = d > 0 ? 1 / d : 0;
            const float *x = w + (size_t)i * cols + g * 32;
            uint8_t *q = p + SCALE_BYTES + g * 64 + i * 16;
            for (int j = 0; j < 16; j++) {
                const int a = (int)lrintf(kb_clamp((x[j] + m) * id, 0, 15));
                const int b = (int)lrintf(kb_clamp((x[j + 16] + m) * id, 0, 15));
                q[j] = (uint8_t)(a | b << 4);
            }
        }
    }
    kb_put6(p + 16, s6);
    kb_put6(p + 40, m6);
}

/* kb_fill_matrix for dtype Q4K (:140-155): 4 rows at a time from one generator stream. */
void or_kb_fill_q4k(int rows, int cols, uint64_t seed, uint8_t *dst) {
    uint64_t s = seed * 0x9E3779B97F4A7C15ull + 7;
    float *w = malloc((size_t)4 * cols * sizeof(float));
    if (!w) abort();
    const size_t tile_bytes = (size_t)(cols / SB_COLS) * SB_BYTES;
    for (int r = 0; r < rows; r += 4) {
        kb_gen(w, (size_t)4 * cols, &s, 0.05f);
        uint8_t *out = dst + (size_t)(r / 4) * tile_bytes;
        for (int sb = 0; sb < cols / SB_COLS; sb++)
            kb_pack_q4k_sb(w + sb * SB_COLS, cols, out + (size_t)sb * SB_BYTES);
    }
    free(w);
}

uint64_t or_fnv1a(const void *p, size_t n) {   /* engine/bench/kbench.c:164-169 */
    const unsigned char *b = p;
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}
