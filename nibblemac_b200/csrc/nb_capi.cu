// Kernel-level C ABI of the Q4K x A8 matmul (include/nb_b200.h): the pf_matmul contract on
// device buffers, for the parity tests and the matvec benchmark.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "nb_b200.h"
#include "nb_dev.cuh"
#include "nb_engine.h"

using namespace nb;

// ------------------------------------------------------------------ allocation-free scratch
// nb_mv_run_static keeps its scratch in this array of the library's own device image instead of
// cudaMalloc'd buffers. Layout: [Step control block, padded to a multiple of 256 B][A8 codes q:
// 16 x 8192 int8][block scales d: 16 x 256 fp32][block sums fsum: 16 x 256 fp32]; kStaticBytes
// per device (pinned below).
namespace {
constexpr int kStaticMaxCols = NB_MV_STATIC_MAX_COLS;
constexpr int kStaticMaxN = NB_MV_STATIC_MAX_N;
static_assert(kStaticMaxN == kMaxRows, "the static scratch holds one full pass of vectors");
static_assert(kStaticMaxCols % 256 == 0, "whole Q4K superblocks");
constexpr size_t kStaticQOff = (sizeof(Step) + 255) & ~(size_t)255;
constexpr size_t kStaticQBytes = (size_t)kStaticMaxN * kStaticMaxCols;
constexpr size_t kStaticDOff = kStaticQOff + kStaticQBytes;
constexpr size_t kStaticDBytes = sizeof(float) * kStaticMaxN * (kStaticMaxCols / 32);
constexpr size_t kStaticFsOff = kStaticDOff + kStaticDBytes;
constexpr size_t kStaticBytes = kStaticFsOff + kStaticDBytes;
constexpr int kStaticMaxDevices = 64;
// The documented size (include/nb_b200.h): a change of the control block's size shows here.
static_assert(kStaticQOff == NB_MV_STATIC_STEP_BYTES, "static scratch: control block size changed");
static_assert(kStaticBytes == NB_MV_STATIC_BYTES, "static scratch: total size changed");

std::mutex g_static_mu;
std::atomic<unsigned char *> g_static_addr[kStaticMaxDevices];
}  // namespace

static __device__ __align__(256) unsigned char g_mv_static_scratch[kStaticBytes];

namespace {
// The scratch's address on the current device, looked up on every call with that device current
// (a cheap table read once the runtime has loaded this library's device image there; the first
// lookup loads it). When the address differs from the one cached for the device (the first call,
// or a primary context torn down by cudaDeviceReset and made anew, which also drops the kernels'
// shared-memory limits), the matvec kernels' shared-memory limits are raised again before use.
unsigned char *static_scratch() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticMaxDevices) {
        set_last_error("nb_mv_run_static: no current CUDA device (or device index >= 64)");
        return nullptr;
    }
    void *addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_mv_static_scratch);
    if (e != cudaSuccess || !addr) {
        char b[200];
        snprintf(b, sizeof b, "nb_mv_run_static: cudaGetSymbolAddress failed on device %d: %s", dev,
                 cudaGetErrorString(e));
        set_last_error(b);
        return nullptr;
    }
    unsigned char *p = static_cast<unsigned char *>(addr);
    if (g_static_addr[dev].load(std::memory_order_acquire) == p) return p;
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_addr[dev].load(std::memory_order_relaxed) == p) return p;
    if (kernels_init(0, 0, 0) != 0) {
        set_last_error("nb_mv_run_static: raising the kernels' shared-memory limits failed");
        return nullptr;
    }
    g_static_addr[dev].store(p, std::memory_order_release);
    return p;
}
}  // namespace

// The device's restated expf / log1pf on an array (the DeltaNet gates' functions), for tests.
__global__ void k_libm_eval(int fn, const float *x, float *y, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = fn == 0 ? glibc_expf(x[i]) : glibc_log1pf(x[i]);
}

struct nb_mv {
    int rows, cols, nmax, n;
    Act act;
    Step *step;
    GemmMaps maps;   // nmax > kMaxRows: TMA descriptors of the activation scratch
    int *status;     // the GEMM's device-wait status word
    uint8_t *tiled;  // nmax > kMaxRows: tile image of the prepared weights (room for 2 x rows)
    GemmW w;         // the prepared weights (nb_mv_prepare)
    float *ypair;    // epilogue 3: gate / up rows [nmax][2 rows]
};

namespace {
Mat panel_mat(const void *W, int rows, int cols) {
    Mat m;
    m.w = (const uint8_t *)W;
    m.rows = rows;
    m.cols = cols;
    m.npanels = (rows + kPanelRows - 1) / kPanelRows;
    m.nsb = cols / 256;
    return m;
}
}  // namespace

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
    if (!nb_q4k_panel_bytes(rows, cols) || nmax < 1 || nmax > NB_MV_MAX_N) return nullptr;
    nb_mv *h = new (std::nothrow) nb_mv();
    if (!h) return nullptr;
    h->rows = rows;
    h->cols = cols;
    h->nmax = nmax;
    h->n = 0;
    h->act.cols = cols;
    const size_t nr = (size_t)std::max(nmax, kMaxRows);
    bool ok = cudaMalloc(&h->act.q, nr * cols) == cudaSuccess &&
              cudaMalloc(&h->act.d, sizeof(float) * nr * (cols / 32)) == cudaSuccess &&
              cudaMalloc(&h->act.fs, sizeof(float) * nr * (cols / 32)) == cudaSuccess &&
              cudaMalloc(&h->step, sizeof(Step)) == cudaSuccess &&
              cudaMemset(h->step, 0, sizeof(Step)) == cudaSuccess &&
              cudaMalloc(&h->status, sizeof(int)) == cudaSuccess &&
              cudaMemset(h->status, 0, sizeof(int)) == cudaSuccess;
    if (!ok) {
        nb_mv_destroy(h);
        return nullptr;
    }
    if (kernels_init(0, 0, 0) != 0) {
        nb_mv_destroy(h);
        return nullptr;
    }
    if (nmax > kMaxRows) {
        const size_t rows2 = (size_t)((rows + 31) / 32) * 32 * 2;
        if (gemm_maps(h->act, (int)nr, &h->maps) != 0 ||
            cudaMalloc(&h->tiled, gemm_tiled_bytes((int)rows2, cols)) != cudaSuccess ||
            cudaMalloc(&h->ypair, sizeof(float) * nr * rows2) != cudaSuccess) {
            nb_mv_destroy(h);
            return nullptr;
        }
    }
    return h;
}

void nb_mv_destroy(nb_mv *h) {
    if (!h) return;
    cudaFree(h->act.q);
    cudaFree(h->act.d);
    cudaFree(h->act.fs);
    cudaFree(h->step);
    cudaFree(h->status);
    cudaFree(h->tiled);
    cudaFree(h->ypair);
    delete h;
}

int nb_mv_set_n(nb_mv *h, int n, void *stream) {
    if (!h || n < 1 || n > h->nmax) return PINFER_E_ARG;
    h->n = n;
    if (n > kMaxRows) return PINFER_OK;   // the tensor-core path takes n as an argument
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
    const Mat m = panel_mat(W, h->rows, h->cols);
    if (h->n > kMaxRows) {   // tcgen05 tiles: widen the weights, then the GEMM
        const int rc = nb_mv_prepare(h, W, nullptr, stream);
        if (rc) return rc;
        return nb_mv_gemm(h, 0, Y, nullptr, nullptr, nullptr, nullptr, nullptr, stream);
    } else {
        launch_matvec(m, h->act, h->step, Y, h->rows, 0, h->nmax, (cudaStream_t)stream);
    }
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_prepare(nb_mv *h, const void *W0, const void *W1, void *stream) {
    if (!h || !W0 || h->nmax <= kMaxRows || (W1 && h->rows % 32)) return PINFER_E_ARG;
    const Mat m0 = panel_mat(W0, h->rows, h->cols);
    Mat m1;
    if (W1) m1 = panel_mat(W1, h->rows, h->cols);
    launch_gemm_tile(m0, m1, h->tiled, (cudaStream_t)stream);
    h->w = gemm_w(m0, m1, h->tiled);
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_gemm(nb_mv *h, int epi, float *Y, void *q, void *d, void *fs, void *partial, int *nan0,
               void *stream) {
    if (!h || !h->w.t || h->n < 1 || h->nmax <= kMaxRows || (epi != 0 && epi != 1 && epi != 3 && epi != 4) ||
        ((epi == 0 || epi == 1) && (!Y || h->w.rows != h->rows)) ||
        (epi == 3 && (!q || !d || !fs || h->w.rows != 2 * h->rows)) ||
        (epi == 4 && (!partial || !nan0 || h->w.rows != h->rows)))
        return PINFER_E_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    GemmArgs g;
    g.W = h->w;
    g.n = h->n;
    g.y = epi == 3 ? h->ypair : Y;
    g.ldy = h->w.rows;
    g.partial = (unsigned long long *)partial;
    g.nan0 = nan0;
    g.status = h->status;
    launch_gemm(epi == 3 ? 0 : epi, h->maps, g, s);
    if (epi == 3) {
        Act out;
        out.q = (int8_t *)q;
        out.d = (float *)d;
        out.fs = (float *)fs;
        out.cols = h->rows;
        launch_swiglu_quant(h->ypair, h->w.rows, h->rows, h->n, out, s);
    }
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

int nb_mv_status(nb_mv *h) {
    int v = 0;
    if (!h || cudaMemcpy(&v, h->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return PINFER_E_ARG;
    return v;
}

int nb_mv_matmul_repeat(nb_mv *h, const void *W, size_t stride, int copies, float *Y, int iters,
                        void *stream) {
    if (!h || !W || !Y || h->n < 1 || copies < 1 || iters < 1) return PINFER_E_ARG;
    for (int i = 0; i < iters; i++) {
        const Mat m = panel_mat((const uint8_t *)W + (size_t)(i % copies) * stride, h->rows, h->cols);
        if (h->n > kMaxRows) {
            const int rc = nb_mv_matmul(h, m.w, Y, stream);
            if (rc) return rc;
        } else {
            launch_matvec(m, h->act, h->step, Y, h->rows, 0, h->nmax, (cudaStream_t)stream);
        }
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

int nb_libm_eval_device(int fn, const float *x, float *y, long long n, void *stream) {
    if ((fn != 0 && fn != 1) || !x || !y || n < 0) return PINFER_E_ARG;
    if (n == 0) return PINFER_OK;
    const long long blocks = std::min<long long>((n + 255) / 256, 4096);
    k_libm_eval<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(fn, x, y, n);
    return cudaGetLastError() == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
}

// The nb_mv_create + nb_mv_set_n + nb_mv_run sequence without an allocation: same kernels, same
// launches, scratch in g_mv_static_scratch. For callers that must not allocate device memory
// during the call: a host whose own caching allocator has already reserved the device's memory
// (a cudaMalloc from the side then fails or fragments that pool), and a host that cannot take
// the device-wide synchronisation cudaMalloc / cudaFree imply while other streams run.
// One scratch per device, so two calls in flight at the same time on one device (other
// streams, other threads) race on it: the caller serialises them.
int nb_mv_run_static(const void *W, int rows, int cols, const float *X, int n, float *Y,
                     void *stream) {
    if (!W || !X || !Y || !nb_q4k_panel_bytes(rows, cols) || n < 1) {
        set_last_error("nb_mv_run_static: null buffer, n < 1, or rows / cols not multiples of 4 / 256");
        return PINFER_E_ARG;
    }
    if (cols > kStaticMaxCols || n > kStaticMaxN) {
        char b[200];
        snprintf(b, sizeof b,
                 "nb_mv_run_static: n=%d cols=%d exceed the static scratch (n <= %d, cols <= %d); "
                 "use nb_mv_create", n, cols, kStaticMaxN, kStaticMaxCols);
        set_last_error(b);
        return PINFER_E_ARG;
    }
    unsigned char *base = static_scratch();
    if (!base) return PINFER_E_NOMEM;
    cudaStream_t s = (cudaStream_t)stream;
    Step *step = reinterpret_cast<Step *>(base);
    Act act;
    act.q = reinterpret_cast<int8_t *>(base + kStaticQOff);
    act.d = reinterpret_cast<float *>(base + kStaticDOff);
    act.fs = reinterpret_cast<float *>(base + kStaticFsOff);
    act.cols = cols;
    // Step::status is the word a kernel sets when a bounded device wait gives up; it must read 0
    // before the launches. The fields the kernels read (n, pos0, logged, tokens) are written by
    // k_set_pass, and the A8 rows 0..n-1 by the quantiser, on every call, so nothing else needs
    // clearing.
    if (cudaMemsetAsync(&step->status, 0, sizeof(int), s) != cudaSuccess) {
        set_last_error("nb_mv_run_static: clearing the status word failed");
        return PINFER_E_NOMEM;
    }
    int tok[kMaxRows] = {0};
    launch_set_pass(step, n, 0, 0, tok, s);
    launch_quant_act(X, n, cols, act, s);
    Mat m;
    m.w = (const uint8_t *)W;
    m.rows = rows;
    m.cols = cols;
    m.npanels = (rows + kPanelRows - 1) / kPanelRows;
    m.nsb = cols / 256;
    launch_matvec(m, act, step, Y, rows, 0, n, s);
    if (cudaGetLastError() != cudaSuccess) {
        set_last_error("nb_mv_run_static: kernel launch failed");
        return PINFER_E_NOMEM;
    }
    // the status word after the launches: a bounded device wait that gave up leaves -90 there
    // and Y incomplete, so the call waits for its stream and reports it
    int status = 0;
    if (cudaMemcpyAsync(&status, &step->status, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        set_last_error("nb_mv_run_static: reading the status word failed");
        return PINFER_E_NOMEM;
    }
    if (status != 0) {
        char b[160];
        snprintf(b, sizeof b, "nb_mv_run_static: a device wait gave up (status %d); Y is not valid", status);
        set_last_error(b);
        return PINFER_E_NOMEM;
    }
    return PINFER_OK;
}

// Test hook: one warp waits on an mbarrier that expects transaction bytes no copy will ever
// bring, with `spin_limit` polls per wait, as every bounded wait of the kernels above does. The
// wait gives up, the warp records -90 in the status word, waits once more (bounded) as the
// kernels do for their copies in flight, and returns; nothing is copied, so nothing is left in
// flight. *status_out receives the status word. 0, or -4 / -3.
static __global__ void k_wait_timeout_probe(int *status, unsigned spin_limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_arrive_expect(&bar, 1024u);   // the one arrival, 1024 bytes that never come
    }
    __syncwarp();
    if (!mbar_wait(&bar, 0, spin_limit)) {
        if (threadIdx.x == 0) *status = -90;
        mbar_wait(&bar, 0, spin_limit);
    }
}

int nb_test_bounded_wait(unsigned spin_limit, int *status_out) {
    if (!status_out || spin_limit == 0 || spin_limit > (1u << 22)) return PINFER_E_ARG;
    int *d = nullptr;
    if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return PINFER_E_NOMEM;
    bool ok = cudaMemset(d, 0, sizeof(int)) == cudaSuccess;
    if (ok) {
        k_wait_timeout_probe<<<1, 32>>>(d, spin_limit);
        ok = cudaGetLastError() == cudaSuccess &&
             cudaMemcpy(status_out, d, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
    }
    cudaFree(d);
    return ok ? PINFER_OK : PINFER_E_NOMEM;
}

}  // extern "C"
