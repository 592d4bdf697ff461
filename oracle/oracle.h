/* CPU oracle for the Q4K x A8 path: TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference engine's quantised matvec arithmetic, used by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker. The product
 * (libpinfer.so) never links or calls it.
 *
 * Why a restatement: the reference's Q4K kernels (engine/src/kern_quant.c, kern_act.c) include
 * <arm_neon.h> unconditionally and cannot be compiled on x86. Every function below cites the
 * reference lines it follows. Compile with -ffp-contract=off: the reference relies on separate
 * multiply / add roundings everywhere except the explicit fused steps (fmaf below), which are
 * exactly the places where its NEON code uses vfmaq / vfmsq.
 *
 * Pinned by: the kbench yhash values the reference recorded on the Pi for the Q4K kernel
 * (FNV-1a of the fp32 outputs for kbench's seeded inputs), tests/golden/kbench_yhash.json. */
#ifndef NB_ORACLE_H
#define NB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-32-column int8 activation quantisation, block-major output:
 * q [cols/32][n][32], d and fsum [cols/32][n]. */
void or_quant_act(const float *X, int n, int cols, int8_t *q, float *d, float *fsum);

/* Y[n][rows] = W x X for a packed Q4K_G32 matrix (the .pq layout). Quantises X internally. */
void or_q4k_matmul(const uint8_t *W, int rows, int cols, const float *X, int n, float *Y);

/* Same, from already-quantised activations (q, d, fsum as or_quant_act writes them). */
void or_q4k_matmul_act(const uint8_t *W, int rows, int cols, const int8_t *q, const float *d,
                       const float *fsum, int n, float *Y);

/* Integer block dot products only: isum[n][rows][cols/32] (int32, exact). */
void or_q4k_isums(const uint8_t *W, int rows, int cols, const int8_t *q, int n, int32_t *isum);

/* One dequantised row (embedding lookup). */
void or_q4k_get_row(const uint8_t *W, int rows, int cols, int row, float *dst);

/* kbench's seeded inputs: a Q4K matrix packed by kbench's simple packer, and the activation
 * vector stream. */
void or_kb_fill_vec(float *x, size_t n, uint64_t seed);
void or_kb_fill_q4k(int rows, int cols, uint64_t seed, uint8_t *dst);

/* 64-bit FNV-1a (kbench's yhash). */
uint64_t or_fnv1a(const void *p, size_t n);

#ifdef __cplusplus
}
#endif
#endif
