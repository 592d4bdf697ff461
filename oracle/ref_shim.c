/* Q4K support for the reference engine's scalar build: TEST INFRASTRUCTURE ONLY.
 *
 * oracle/Makefile compiles the reference engine's own sources (engine/src/*.c, MATVEC=ref)
 * unmodified into oracle/_ref/. Its scalar kernel file matvec_ref.c handles only F32 / BF16
 * (engine/src/matvec_ref.c:43) and the Q4K kernels are NEON-only, so matvec_ref.c is compiled
 * with its four dispatch entry points renamed (*_scalar, the same -D trick as
 * engine/macos/Makefile:50-51) and this file provides the public names: dtype Q4K_G32 goes to
 * the restatement in q4k_a8.c (pinned by the reference's recorded kbench hashes), everything
 * else to the reference's own scalar code. */
#include <stdint.h>
#include <stdlib.h>

#include "ops.h"
#include "oracle.h"

#define Q4K 4u

void pf_matmul_scalar(pf_pool *pool, const pf_mat *W, const float *X, float *Y, int n);
void pf_matvec_scalar(pf_pool *pool, const pf_mat *W, const float *x, float *y);
void pf_get_row_scalar(const pf_mat *W, int row, float *dst);
int pf_dtype_supported_scalar(uint32_t dtype);

void pf_matmul(pf_pool *pool, const pf_mat *W, const float *X, float *Y, int n) {
    if (W->dtype != Q4K) {
        pf_matmul_scalar(pool, W, X, Y, n);
        return;
    }
    if (n <= 0) return;
    or_q4k_matmul((const uint8_t *)W->data, W->rows, W->cols, X, n, Y);
}

void pf_matvec(pf_pool *pool, const pf_mat *W, const float *x, float *y) {
    if (W->dtype != Q4K) {
        pf_matvec_scalar(pool, W, x, y);
        return;
    }
    or_q4k_matmul((const uint8_t *)W->data, W->rows, W->cols, x, 1, y);
}

void pf_get_row(const pf_mat *W, int row, float *dst) {
    if (W->dtype != Q4K) {
        pf_get_row_scalar(W, row, dst);
        return;
    }
    or_q4k_get_row((const uint8_t *)W->data, W->rows, W->cols, row, dst);
}

int pf_dtype_supported(uint32_t dtype) {
    return dtype == Q4K || pf_dtype_supported_scalar(dtype);
}
