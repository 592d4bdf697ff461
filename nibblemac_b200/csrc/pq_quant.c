/* Q4K_G32 quantiser and packer for the .pq format (host tool, not on the device path).
 *
 * A C restatement of the reference's numpy quantiser, tools/quant.py quant_asym4 (:78-105),
 * quant_q4k (:108-141), _pack6 (:210-217) and pack_q4k (:220-244), producing the same bytes:
 * every step below is the float32 operation numpy performs, in numpy's order. Two details
 * matter for bit-identity:
 *   - float32 sums over a 32-element group (x.sum(-1) etc.) follow numpy's pairwise summation
 *     for a contiguous run of 8..128 elements: 8 running partial sums r[j] += a[i + j], then
 *     ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7));
 *   - fp16 rounding (.astype(np.float16)) is IEEE round-to-nearest-even.
 * Built with -ffp-contract=off so no multiply-add is fused. tests/test_pq_quant.py checks the
 * output against fixtures made by the reference's own quant.py. */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float f16r(float x) { return (float)(_Float16)x; }   /* .astype(float16).astype(float32) */

static uint16_t f16bits(float x) {
    _Float16 h = (_Float16)x;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

/* numpy pairwise_sum for n = 32 contiguous float32 values */
static float psum32(const float *a) {
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    for (int i = 8; i < 32; i += 8)
        for (int j = 0; j < 8; j++) r[j] = r[j] + a[i + j];
    return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
}

static float clipf(float v, float lo, float hi) {   /* np.clip (NaN passes through) */
    return v < lo ? lo : v > hi ? hi : v;
}

/* quant_asym4(w, 32, iters=4) for one group of 32: the fp16-rounded scale d16 and min m16. */
static void asym4_group(const float *x, float *d16_out, float *m16_out) {
    float lo = x[0], hi = x[0];
    for (int j = 1; j < 32; j++) {
        lo = x[j] < lo ? x[j] : lo;
        hi = x[j] > hi ? x[j] : hi;
    }
    float d = (hi - lo) / 15.0f, m = lo, d16 = 0, m16 = 0;
    float q[32], t[32];
    for (int it = 0; it <= 4; it++) {
        d16 = f16r(d);
        m16 = f16r(m);
        const float safe = d16 == 0.0f ? 1.0f : d16;
        for (int j = 0; j < 32; j++) q[j] = clipf(rintf((x[j] - m16) / safe), 0.0f, 15.0f);
        if (it == 4) break;
        const float n = 32.0f;
        const float sq = psum32(q), sx = psum32(x);
        for (int j = 0; j < 32; j++) t[j] = q[j] * q[j];
        const float sqq = psum32(t);
        for (int j = 0; j < 32; j++) t[j] = q[j] * x[j];
        const float sqx = psum32(t);
        const float den = n * sqq - sq * sq;
        const int ok = den > 0.0f;
        const float dn = ok ? (n * sqx - sq * sx) / den : d;
        const float mn = ok ? (sx - dn * sq) / n : m;
        d = dn;
        m = mn;
    }
    *d16_out = d16;
    *m16_out = m16;
}

/* 32 values in [0, 63] -> 24 bytes (quant.py _pack6) */
static void pack6(const uint8_t *v, uint8_t *p) {
    for (int i = 0; i < 16; i++) p[i] = (uint8_t)((v[i] & 15) | ((v[i + 16] & 15) << 4));
    for (int i = 0; i < 8; i++)
        p[16 + i] = (uint8_t)((v[i] >> 4) | ((v[i + 8] >> 4) << 2) | ((v[i + 16] >> 4) << 4) |
                              ((v[i + 24] >> 4) << 6));
}

/* quant_q4k for one row's superblock (256 columns, 8 groups) given the groups' asym4 fits:
 * writes D, M (fp16-rounded) and the 6-bit s, m and 4-bit codes. */
static void q4k_row_sb(const float *x, float *D_out, float *M_out, uint8_t *s_out,
                       uint8_t *m_out, uint8_t *q_out) {
    float dg[8], mn[8];
    for (int g = 0; g < 8; g++) {
        float d16, m16;
        asym4_group(x + 32 * g, &d16, &m16);
        dg[g] = d16;
        const float neg = -m16;
        mn[g] = neg > 0.0f ? neg : (neg != neg ? neg : 0.0f);   /* np.maximum(-mg, 0) */
    }
    float dmax = dg[0], mmax = mn[0];
    for (int g = 1; g < 8; g++) {
        dmax = dg[g] > dmax ? dg[g] : dmax;
        mmax = mn[g] > mmax ? mn[g] : mmax;
    }
    const float D = f16r(dmax / 63.0f), M = f16r(mmax / 63.0f);
    const float Ds = D == 0.0f ? 1.0f : D, Ms = M == 0.0f ? 1.0f : M;
    float sq[8], mq[8], q[32], t[32];
    for (int g = 0; g < 8; g++) {
        sq[g] = clipf(rintf(dg[g] / Ds), 0.0f, 63.0f);
        mq[g] = clipf(rintf(mn[g] / Ms), 0.0f, 63.0f);
    }
    for (int g = 0; g < 8; g++) {
        const float *xg = x + 32 * g;
        for (int it = 0; it <= 2; it++) {
            const float d_eff = D * sq[g], m_eff = M * mq[g];
            const float safe = d_eff == 0.0f ? 1.0f : d_eff;
            for (int j = 0; j < 32; j++) q[j] = clipf(rintf((xg[j] + m_eff) / safe), 0.0f, 15.0f);
            if (it == 2) break;
            const float n = 32.0f;
            const float s_q = psum32(q), sx = psum32(xg);
            for (int j = 0; j < 32; j++) t[j] = q[j] * q[j];
            const float sqq = psum32(t);
            for (int j = 0; j < 32; j++) t[j] = q[j] * xg[j];
            const float sqx = psum32(t);
            const float den = n * sqq - s_q * s_q;
            const int ok = den > 0.0f;
            const float dn = ok ? (n * sqx - s_q * sx) / den : d_eff;
            const float mm = ok ? -(sx - dn * s_q) / n : m_eff;
            sq[g] = clipf(rintf(dn / Ds), 0.0f, 63.0f);
            const float mpos = mm > 0.0f ? mm : (mm != mm ? mm : 0.0f);
            mq[g] = clipf(rintf(mpos / Ms), 0.0f, 63.0f);
        }
        for (int j = 0; j < 32; j++) q_out[32 * g + j] = (uint8_t)q[j];
        s_out[g] = (uint8_t)sq[g];
        m_out[g] = (uint8_t)mq[g];
    }
    *D_out = D;
    *M_out = M;
}

/* Quantise + pack rows [t0*4, t1*4) of W [rows][cols] (float32) into `out` (the packed
 * matrix, tile t at t * cols/256 * 576). */
static void pack_tiles(const float *W, int cols, int t0, int t1, uint8_t *out) {
    const int nsb = cols / 256;
    for (int t = t0; t < t1; t++)
        for (int sb = 0; sb < nsb; sb++) {
            uint8_t *p = out + ((size_t)t * nsb + sb) * 576;
            uint8_t s6[32], m6[32], codes[4][256];
            for (int i = 0; i < 4; i++) {
                float D, M;
                uint8_t s[8], m[8];
                q4k_row_sb(W + (size_t)(4 * t + i) * cols + 256 * sb, &D, &M, s, m, codes[i]);
                const uint16_t hd = f16bits(D), hm = f16bits(M);
                memcpy(p + 2 * i, &hd, 2);
                memcpy(p + 8 + 2 * i, &hm, 2);
                for (int g = 0; g < 8; g++) {   /* [group][row] order */
                    s6[4 * g + i] = s[g];
                    m6[4 * g + i] = m[g];
                }
            }
            pack6(s6, p + 16);
            pack6(m6, p + 40);
            for (int g = 0; g < 8; g++)
                for (int i = 0; i < 4; i++) {
                    uint8_t *c = p + 64 + 64 * g + 16 * i;
                    for (int j = 0; j < 16; j++)
                        c[j] = (uint8_t)(codes[i][32 * g + j] | (codes[i][32 * g + 16 + j] << 4));
                }
        }
}

/* Exported: quantise and pack a [rows][cols] float32 matrix (rows % 4 == 0, cols % 256 == 0)
 * into rows/4 * cols/256 * 576 bytes. Returns 0, or -1 for a bad shape. Row tiles are
 * independent, so the work is split over threads without changing any byte. */
int nb_q4k_quantize_pack(const float *W, int rows, int cols, uint8_t *out, int nthreads) {
    if (rows <= 0 || cols <= 0 || rows % 4 || cols % 256) return -1;
    const int tiles = rows / 4;
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 16)
    for (int t = 0; t < tiles; t++) pack_tiles(W, cols, t, t + 1, out);
    return 0;
}
