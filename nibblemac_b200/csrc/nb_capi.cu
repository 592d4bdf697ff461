// Kernel-level C ABI of the Q4K x A8 matmul (include/nb_b200.h): the pf_matmul contract on
// device buffers, for the parity tests and the matvec benchmark.
#include <cstring>
#include <new>

#include "nb_b200.h"
#include "nb_engine.h"

using namespace nb;

struct nb_mv {
    int rows, cols, nmax, n;
    Act act;
    Step *step;
};

extern "C" {

size_t nb_q4k_panel_bytes(int rows, int cols) {
    if (rows <= 0 || cols <= 0 || rows % 4 || cols % 256) return 0;
    return panel_bytes(rows, cols);
}

int nb_q4k_repack(const uint8_t *pq, int rows, int cols, uint8_t *panels) {
    if (!pq || !panels || !nb_q4k_panel_bytes(rows, cols)) return PINFER_E_ARG;
    repack_q4k(pq, rows, cols, panels);
    return PINFER_OK;
}

nb_mv *nb_mv_create(int rows, int cols, int nmax) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1) return nullptr;
    if (!nb_q4k_panel_bytes(rows, cols) || nmax < 1 || nmax > kMaxRows) return nullptr;
    nb_mv *h = new (std::nothrow) nb_mv();
    if (!h) return nullptr;
    h->rows = rows;
    h->cols = cols;
    h->nmax = nmax;
    h->n = 0;
    h->act.cols = cols;
    bool ok = cudaMalloc(&h->act.q, (size_t)kMaxRows * cols) == cudaSuccess &&
              cudaMalloc(&h->act.d, sizeof(float) * kMaxRows * (cols / 32)) == cudaSuccess &&
              cudaMalloc(&h->act.fs, sizeof(float) * kMaxRows * (cols / 32)) == cudaSuccess &&
              cudaMalloc(&h->step, sizeof(Step)) == cudaSuccess &&
              cudaMemset(h->step, 0, sizeof(Step)) == cudaSuccess;
    if (!ok) {
        nb_mv_destroy(h);
        return nullptr;
    }
    if (kernels_init(0, 0, 0) != 0) {
        nb_mv_destroy(h);
        return nullptr;
    }
    return h;
}

void nb_mv_destroy(nb_mv *h) {
    if (!h) return;
    cudaFree(h->act.q);
    cudaFree(h->act.d);
    cudaFree(h->act.fs);
    cudaFree(h->step);
    delete h;
}

int nb_mv_set_n(nb_mv *h, int n, void *stream) {
    if (!h || n < 1 || n > h->nmax) return PINFER_E_ARG;
    h->n = n;
    int tok[kMaxRows] = {0};
    launch_set_pass(h->step, n, 0, 0, tok, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_quant(nb_mv *h, const float *X, void *stream) {
    if (!h || !X || h->n < 1) return PINFER_E_ARG;
    launch_quant_act(X, h->n, h->cols, h->act, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_matmul(nb_mv *h, const void *W, float *Y, void *stream) {
    if (!h || !W || !Y || h->n < 1) return PINFER_E_ARG;
    Mat m;
    m.w = (const uint8_t *)W;
    m.rows = h->rows;
    m.cols = h->cols;
    m.npanels = (h->rows + kPanelRows - 1) / kPanelRows;
    m.nsb = h->cols / 256;
    launch_matvec(m, h->act, h->step, Y, h->rows, 0, h->nmax, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_matmul_repeat(nb_mv *h, const void *W, size_t stride, int copies, float *Y, int iters,
                        void *stream) {
    if (!h || !W || !Y || h->n < 1 || copies < 1 || iters < 1) return PINFER_E_ARG;
    Mat m;
    m.rows = h->rows;
    m.cols = h->cols;
    m.npanels = (h->rows + kPanelRows - 1) / kPanelRows;
    m.nsb = h->cols / 256;
    for (int i = 0; i < iters; i++) {
        m.w = (const uint8_t *)W + (size_t)(i % copies) * stride;
        launch_matvec(m, h->act, h->step, Y, h->rows, 0, h->nmax, (cudaStream_t)stream);
    }
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_head_repeat(nb_mv *h, const void *W, size_t stride, int copies, float *Y, int iters,
                      void *partial, int *nan0, void *stream) {
    if (!h || !W || h->n < 1 || copies < 1 || iters < 1 || !partial || !nan0) return PINFER_E_ARG;
    Mat m;
    m.rows = h->rows;
    m.cols = h->cols;
    m.npanels = (h->rows + kPanelRows - 1) / kPanelRows;
    m.nsb = h->cols / 256;
    for (int i = 0; i < iters; i++) {
        m.w = (const uint8_t *)W + (size_t)(i % copies) * stride;
        launch_matvec_head(m, h->act, h->step, Y, h->rows, (unsigned long long *)partial, nan0,
                           h->nmax, (cudaStream_t)stream);
    }
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_run(nb_mv *h, const void *W, const float *X, float *Y, void *stream) {
    const int rc = nb_mv_quant(h, X, stream);
    return rc ? rc : nb_mv_matmul(h, W, Y, stream);
}

int nb_mv_get_act(nb_mv *h, int8_t *q, float *d, float *fsum, void *stream) {
    if (!h || !q || !d || !fsum || h->n < 1) return PINFER_E_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t nb = (size_t)h->n * (h->cols / 32);
    bool ok = cudaMemcpyAsync(q, h->act.q, (size_t)h->n * h->cols, cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
              cudaMemcpyAsync(d, h->act.d, nb * 4, cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
              cudaMemcpyAsync(fsum, h->act.fs, nb * 4, cudaMemcpyDeviceToDevice, s) == cudaSuccess;
    return ok ? PINFER_OK : PINFER_E_NOMEM;
}

}  // extern "C"
