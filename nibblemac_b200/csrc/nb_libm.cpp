// Host-side checks of the restated glibc expf / log1pf (nb_math.cuh), which the device uses
// for the Gated DeltaNet gates (engine/src/forward_lin.c:19,290-293).
//
// nb_libm_selftest compares the restatements, compiled for the host from the same source the
// device uses, with the C library's own expf and log1pf on every `stride`-th 32-bit pattern
// (stride 1: all 2^32 inputs, NaN results compared as NaN). nb_libm_eval_host returns the C
// library's values, so a GPU test can compare the device's evaluation input by input.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "nb_engine.h"

namespace {

// The C library's functions, called through pointers so the compiler cannot fold or replace them.
float (*volatile g_expf)(float) = expf;
float (*volatile g_log1pf)(float) = log1pf;

inline bool same(float a, float b) {
    return nb::libm_f2u(a) == nb::libm_f2u(b) || (std::isnan(a) && std::isnan(b));
}

}  // namespace

extern "C" {

// Mismatches between restatement and C library over inputs i * stride (i >= 0, < 2^32), both
// functions, `threads` host threads. Returns 0 (count in *mismatches) or -1 on bad arguments.
int nb_libm_selftest(int threads, long long stride, long long *mismatches) {
    if (threads < 1 || stride < 1 || !mismatches) return -1;
    std::vector<long long> bad(threads, 0);
    std::vector<std::thread> pool;
    const uint64_t n = (0x100000000ull + (uint64_t)stride - 1) / (uint64_t)stride;
    for (int t = 0; t < threads; t++) {
        pool.emplace_back([&, t] {
            long long b = 0;
            for (uint64_t i = t; i < n; i += threads) {
                const float x = nb::libm_u2f((uint32_t)(i * (uint64_t)stride));
                if (!same(nb::glibc_expf(x), g_expf(x))) b++;
                if (!same(nb::glibc_log1pf(x), g_log1pf(x))) b++;
            }
            bad[t] = b;
        });
    }
    for (auto &th : pool) th.join();
    long long total = 0;
    for (long long b : bad) total += b;
    *mismatches = total;
    return 0;
}

// y[i] = expf(x[i]) (fn 0) or log1pf(x[i]) (fn 1) from the C library (host arrays).
int nb_libm_eval_host(int fn, const float *x, float *y, long long n) {
    if ((fn != 0 && fn != 1) || !x || !y || n < 0) return -1;
    for (long long i = 0; i < n; i++) y[i] = fn == 0 ? g_expf(x[i]) : g_log1pf(x[i]);
    return 0;
}

// The argmax key of (v, row) as the device computes it (for host-side checks of the merge).
unsigned long long nb_argmax_key(float v, int row) { return nb::argmax_key(v, row); }

}  // extern "C"
