// Host-side tables that let the device reproduce glibc's expf / log1pf bit for bit.
//
// The reference computes the Gated DeltaNet gates with glibc's expf and log1pf
// (engine/src/forward_lin.c:19,288-293). glibc's results differ from the correctly rounded
// value by one ulp for a small fraction of inputs (measured here: ~5e-5 for expf, ~1.5% for
// log1pf), and the greedy tokens depend on those bits. The device computes the correctly
// rounded value in double precision; this file builds, by calling glibc's own functions on
// every input of the domain, a 2-bit code per input:
//   0 glibc == round(double result)   1 glibc is one ulp above   2 one ulp below
//   3 the double result is within 2^-46 (relative) of a float rounding boundary, so another
//     double implementation might round it differently: glibc's value is kept in a sorted
//     overflow list instead.
// Domains: expf for 2^-30 <= |x| <= 104, log1pf for 2^-30 <= y <= 4.866e8 (> expf(20)); the
// two functions agree with the rounded double results outside them (checked by tests).
// The tables take ~280 MB and a few seconds of host time; they are cached in a file.
#include <dlfcn.h>
#include <gnu/libc-version.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "nb_engine.h"

namespace nb {
namespace {

constexpr uint32_t kMagic = 0x4e424c4du;   // "NBLM"
constexpr uint32_t kFormat = 2;

inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

// The glibc functions, called through pointers so the compiler cannot fold or replace them.
float (*volatile g_expf)(float) = expf;
float (*volatile g_log1pf)(float) = log1pf;
double (*volatile g_exp)(double) = exp;
double (*volatile g_log1p)(double) = log1p;

// Code of one input: `g` glibc's float result, `dd` the double-precision result.
inline uint32_t code_of(float g, double dd, bool *ambiguous) {
    const float c = (float)dd;
    *ambiguous = false;
    if (std::isfinite(c) && std::isfinite(dd) && c != 0.0f) {
        const float nb = dd > (double)c ? nextafterf(c, INFINITY) : nextafterf(c, -INFINITY);
        if (std::isfinite(nb)) {
            const double mid = ((double)c + (double)nb) * 0.5;
            const double scale = std::max(std::fabs(dd), 1.1754943508222875e-38);
            if (std::fabs(dd - mid) <= scale * 0x1p-46) *ambiguous = true;
        }
    }
    if (*ambiguous) return 3u;
    const int64_t delta = (int64_t)f2u(g) - (int64_t)f2u(c);
    if (delta == 0) return 0u;
    if (delta == 1) return 1u;
    if (delta == -1) return 2u;
    *ambiguous = true;   // never seen; kept exact through the overflow list
    return 3u;
}

struct Ovf {
    uint32_t fn, bits;
    float val;
};

// Fill codes for inputs [i0, i1) (multiples of 16, so threads own whole words).
void fill_exp(uint32_t *words, uint64_t i0, uint64_t i1, std::vector<Ovf> *ovf) {
    for (uint64_t i = i0; i < i1; i += 16) {
        uint32_t w = 0;
        for (uint64_t k = 0; k < 16 && i + k < i1; k++) {
            const uint64_t idx = i + k;
            const uint32_t sign = idx >= kExpSpan ? 0x80000000u : 0u;
            const uint32_t b = sign | (kLibmLo + (uint32_t)(idx % kExpSpan));
            const float x = u2f(b);
            bool amb;
            const float g = g_expf(x);
            const uint32_t code = code_of(g, g_exp((double)x), &amb);
            if (amb) ovf->push_back({0u, b, g});
            w |= code << (2 * k);
        }
        words[i >> 4] = w;
    }
}

void fill_log1p(uint32_t *words, uint64_t i0, uint64_t i1, std::vector<Ovf> *ovf) {
    for (uint64_t i = i0; i < i1; i += 16) {
        uint32_t w = 0;
        for (uint64_t k = 0; k < 16 && i + k < i1; k++) {
            const uint32_t b = kLibmLo + (uint32_t)(i + k);
            const float y = u2f(b);
            bool amb;
            const float g = g_log1pf(y);
            const uint32_t code = code_of(g, g_log1p((double)y), &amb);
            if (amb) ovf->push_back({1u, b, g});
            w |= code << (2 * k);
        }
        words[i >> 4] = w;
    }
}

// A fingerprint of this process's glibc: version plus a hash of results on probe inputs, so a
// cache made by another libm (or another CPU dispatch of it) is never used.
uint64_t libm_fingerprint() {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](uint32_t v) { for (int i = 0; i < 4; i++) { h ^= (v >> (8 * i)) & 0xff; h *= 1099511628211ull; } };
    for (const char *p = gnu_get_libc_version(); *p; p++) { h ^= (unsigned char)*p; h *= 1099511628211ull; }
    uint32_t s = 12345;
    for (int i = 0; i < 4096; i++) {
        s = s * 1664525u + 1013904223u;
        const float x = u2f(0x30800000u + s % (kExpHiBits - kLibmLo));
        mix(f2u(g_expf(x)));
        mix(f2u(g_expf(-x)));
        mix(f2u(g_log1pf(x)));
    }
    mix(kFormat);
    return h;
}

std::string cache_path(uint64_t fp) {
    const char *dir = getenv("NB_LIBM_CACHE_DIR");
    std::string d = dir && *dir ? dir : "/tmp";
    char name[96];
    snprintf(name, sizeof name, "/nibblemac_b200_libm_%016llx.tbl", (unsigned long long)fp);
    return d + name;
}

bool read_cache(const std::string &path, uint64_t fp, HostLibm *t) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    uint32_t hdr[2];
    uint64_t hfp, sizes[3];
    bool ok = fread(hdr, 4, 2, f) == 2 && hdr[0] == kMagic && hdr[1] == kFormat &&
              fread(&hfp, 8, 1, f) == 1 && hfp == fp && fread(sizes, 8, 3, f) == 3 &&
              sizes[0] == t->exp_words && sizes[1] == t->log1p_words && sizes[2] < (1u << 24);
    if (ok) {
        t->n_ovf = (int)sizes[2];
        t->ovf_key = (uint32_t *)malloc(sizeof(uint32_t) * 2 * (t->n_ovf + 1));
        t->ovf_val = (float *)malloc(sizeof(float) * (t->n_ovf + 1));
        ok = t->ovf_key && t->ovf_val &&
             fread(t->exp_bits, 4, t->exp_words, f) == t->exp_words &&
             fread(t->log1p_bits, 4, t->log1p_words, f) == t->log1p_words &&
             fread(t->ovf_key, 4, 2 * (size_t)t->n_ovf, f) == 2 * (size_t)t->n_ovf &&
             fread(t->ovf_val, 4, t->n_ovf, f) == (size_t)t->n_ovf;
    }
    fclose(f);
    return ok;
}

void write_cache(const std::string &path, uint64_t fp, const HostLibm *t) {
    const std::string tmp = path + ".tmp" + std::to_string(getpid());
    FILE *f = fopen(tmp.c_str(), "wb");
    if (!f) return;
    const uint32_t hdr[2] = {kMagic, kFormat};
    const uint64_t sizes[3] = {t->exp_words, t->log1p_words, (uint64_t)t->n_ovf};
    bool ok = fwrite(hdr, 4, 2, f) == 2 && fwrite(&fp, 8, 1, f) == 1 && fwrite(sizes, 8, 3, f) == 3 &&
              fwrite(t->exp_bits, 4, t->exp_words, f) == t->exp_words &&
              fwrite(t->log1p_bits, 4, t->log1p_words, f) == t->log1p_words &&
              fwrite(t->ovf_key, 4, 2 * (size_t)t->n_ovf, f) == 2 * (size_t)t->n_ovf &&
              fwrite(t->ovf_val, 4, t->n_ovf, f) == (size_t)t->n_ovf;
    ok = fclose(f) == 0 && ok;
    if (ok) rename(tmp.c_str(), path.c_str());
    else unlink(tmp.c_str());
}

}  // namespace

int libm_tables_get(HostLibm *t, int threads, char *err, size_t errlen) {
    const uint64_t n_exp = 2ull * kExpSpan;
    const uint64_t n_log = (uint64_t)(kLog1pHiBits - kLibmLo) + 1;
    t->exp_words = (size_t)((n_exp + 15) / 16);
    t->log1p_words = (size_t)((n_log + 15) / 16);
    t->exp_bits = (uint32_t *)malloc(t->exp_words * 4);
    t->log1p_bits = (uint32_t *)malloc(t->log1p_words * 4);
    if (!t->exp_bits || !t->log1p_bits) {
        snprintf(err, errlen, "libm tables: out of host memory");
        return -3;
    }
    const uint64_t fp = libm_fingerprint();
    const std::string path = cache_path(fp);
    if (read_cache(path, fp, t)) return 0;
    free(t->ovf_key);
    free(t->ovf_val);
    if (threads < 1) threads = 1;
    std::vector<std::vector<Ovf>> ovf((size_t)threads * 2);
    std::vector<std::thread> pool;
    for (int w = 0; w < threads; w++) {
        pool.emplace_back([&, w] {
            const uint64_t e0 = n_exp * w / threads / 16 * 16, e1 = w + 1 == threads ? n_exp : n_exp * (w + 1) / threads / 16 * 16;
            fill_exp(t->exp_bits, e0, e1, &ovf[2 * w]);
            const uint64_t l0 = n_log * w / threads / 16 * 16, l1 = w + 1 == threads ? n_log : n_log * (w + 1) / threads / 16 * 16;
            fill_log1p(t->log1p_bits, l0, l1, &ovf[2 * w + 1]);
        });
    }
    for (auto &th : pool) th.join();
    std::vector<Ovf> all;
    for (auto &v : ovf) all.insert(all.end(), v.begin(), v.end());
    std::sort(all.begin(), all.end(), [](const Ovf &a, const Ovf &b) {
        return a.fn != b.fn ? a.fn < b.fn : a.bits < b.bits;
    });
    t->n_ovf = (int)all.size();
    t->ovf_key = (uint32_t *)malloc(sizeof(uint32_t) * 2 * (all.size() + 1));
    t->ovf_val = (float *)malloc(sizeof(float) * (all.size() + 1));
    if (!t->ovf_key || !t->ovf_val) {
        snprintf(err, errlen, "libm tables: out of host memory");
        return -3;
    }
    for (size_t i = 0; i < all.size(); i++) {
        t->ovf_key[2 * i] = all[i].fn;
        t->ovf_key[2 * i + 1] = all[i].bits;
        t->ovf_val[i] = all[i].val;
    }
    write_cache(path, fp, t);
    return 0;
}

void libm_tables_free(HostLibm *t) {
    free(t->exp_bits);
    free(t->log1p_bits);
    free(t->ovf_key);
    free(t->ovf_val);
    *t = HostLibm();
}

}  // namespace nb

// Test hooks (C ABI): build the tables on the host and query them like the device does.
extern "C" int nb_libm_selftest(int threads, long long samples, long long *mismatches) {
    nb::HostLibm t;
    char err[128];
    if (nb::libm_tables_get(&t, threads, err, sizeof err)) return -1;
    long long bad = 0;
    uint32_t s = 99;
    for (long long i = 0; i < samples; i++) {
        s = s * 1664525u + 1013904223u;
        const uint32_t r2 = s * 2654435761u;
        const float x = nb::u2f(((s >> 1) % 0x43000000u) | ((r2 & 1u) << 31));
        // expf path
        {
            const uint32_t b = nb::f2u(x), a = b & 0x7fffffffu;
            float c = (float)exp((double)x);
            if (a >= nb::kLibmLo && a <= nb::kExpHiBits) {
                const uint32_t idx = (b >> 31) * nb::kExpSpan + (a - nb::kLibmLo);
                const uint32_t code = (t.exp_bits[idx >> 4] >> ((idx & 15) * 2)) & 3;
                if (code == 1) c = nb::u2f(nb::f2u(c) + 1);
                else if (code == 2) c = nb::u2f(nb::f2u(c) - 1);
                else if (code == 3) {
                    for (int k = 0; k < t.n_ovf; k++)
                        if (t.ovf_key[2 * k] == 0 && t.ovf_key[2 * k + 1] == b) c = t.ovf_val[k];
                }
            }
            if (nb::f2u(c) != nb::f2u(expf(x)) && !(std::isnan(c) && std::isnan(expf(x)))) bad++;
        }
        // log1pf path, y >= 0
        {
            const float y = fabsf(x);
            const uint32_t b = nb::f2u(y);
            float c = (float)log1p((double)y);
            if (b >= nb::kLibmLo && b <= nb::kLog1pHiBits) {
                const uint32_t code = (t.log1p_bits[(b - nb::kLibmLo) >> 4] >> (((b - nb::kLibmLo) & 15) * 2)) & 3;
                if (code == 1) c = nb::u2f(nb::f2u(c) + 1);
                else if (code == 2) c = nb::u2f(nb::f2u(c) - 1);
                else if (code == 3) {
                    for (int k = 0; k < t.n_ovf; k++)
                        if (t.ovf_key[2 * k] == 1 && t.ovf_key[2 * k + 1] == b) c = t.ovf_val[k];
                }
            }
            if (y <= 4.866e8f && nb::f2u(c) != nb::f2u(log1pf(y))) bad++;
        }
    }
    *mismatches = bad;
    const int n_ovf = t.n_ovf;
    nb::libm_tables_free(&t);
    return n_ovf;
}
