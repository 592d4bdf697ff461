/* Synthetic-drafter speculative decoding on the reference engine: TEST INFRASTRUCTURE ONLY.
 *
 * Compiled into oracle/_ref/libpinfer_ref.so together with the reference's unmodified
 * sources. It drives the reference's own internals exactly as pf_spec_decode does
 * (engine/src/spec.c:256-383), steps 2-3 (verify, accept, commit), with the drafts of step 1
 * replaced by the synthetic drafter of the benchmark (no MTP head, no n-gram, fixed k):
 *   verify:  ctx->lin_log_on = 1; pf_forward_h(ctx, vt, ke + 1, ...) (spec.c:323-335)
 *   accept:  longest prefix with vt[i+1] == argmax(logits[i]) plus the bonus (spec.c:339-346)
 *   commit:  pf_lin_commit(ctx, e); n_past = P + e; cur = vt[e] (spec.c:347-350)
 *   end:     pf_lin_flush (spec.c:376)
 * The drafter is the pure function nb_synth_draft below (the device engine implements the same
 * function), so both sides draft the same tokens. */
#define _POSIX_C_SOURCE 200809L
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "forward.h"
#include "pinfer.h"

/* splitmix64 output function */
static uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* Draft for output index j: with probability p24 / 2^24 the target's greedy token at j
 * (greedy[j]), otherwise a uniform token of [0, vocab). */
int32_t nb_synth_draft(uint64_t seed, int64_t j, uint32_t p24, int32_t vocab, int32_t greedy_j) {
    const uint64_t h = mix64(seed ^ mix64((uint64_t)j));
    if ((uint32_t)(h >> 40) < p24) return greedy_j;
    return (int32_t)(mix64(h) % (uint64_t)vocab);
}

static int64_t now_ns(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (int64_t)ts.tv_sec * 1000000000 + ts.tv_nsec;
}

/* stats (may be NULL): [0] rounds, [1] drafted, [2] accepted, [3] ns spent after the prompt
 * (the decode loop, for the benchmark's CPU baseline). greedy: the plain greedy
 * output of the same prompt, n_max entries. append: keep the context and feed the prompt on
 * top of it (pinfer_generate_greedy_cont's rule), else start from a reset context. Returns
 * tokens written or a negative code. */
static int spec_generate(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt, int32_t *out,
                         int n_max, int k, const int32_t *greedy, uint64_t seed, uint32_t p24,
                         int64_t *stats, int append) {
    if (!ctx || !prompt || n_prompt <= 0 || !out || n_max <= 0 || k < 0 ||
        k > PINFER_SPEC_MAX_K || !greedy)
        return PINFER_E_ARG;
    const int V = ctx->vocab;
    float *logits = malloc((size_t)(k + 1) * V * sizeof(float));
    if (!logits) return PINFER_E_NOMEM;
    if (!append) pinfer_reset(ctx);
    int rc = k > 0 ? pf_lin_log_alloc(ctx, k + 1) : PINFER_OK;
    if (rc == PINFER_OK) rc = pf_forward(ctx, prompt, n_prompt, logits, NULL, NULL);
    if (rc != PINFER_OK) {
        free(logits);
        return rc;
    }
    int32_t cur = pinfer_argmax(logits, V), vt[PINFER_SPEC_MAX_K + 2];
    int count = 0;
    out[count++] = cur;
    const int batch = ctx->batch;
    const int64_t t0 = now_ns();
    while (count < n_max) {
        const int P = ctx->n_past;
        int left = n_max - count - 1;
        if (left > ctx->max_ctx - P - 1) left = ctx->max_ctx - P - 1;
        if (left < 0) { rc = PINFER_E_CTX_FULL; break; }
        const int ke = k < left ? k : left;
        if (stats) stats[0]++;
        if (ke == 0) {   /* plain step (spec.c plain_step) */
            rc = pf_forward(ctx, &cur, 1, logits, NULL, NULL);
            if (rc != PINFER_OK) break;
            cur = pinfer_argmax(logits, V);
            out[count++] = cur;
            continue;
        }
        vt[0] = cur;
        for (int s = 1; s <= ke; s++) {
            const int64_t j = count - 1 + s;
            vt[s] = nb_synth_draft(seed, j, p24, V, greedy[j]);
        }
        ctx->lin_log_on = 1;
        if (batch < ke + 1) pf_set_batch(ctx, ke + 1);
        rc = pf_forward_h(ctx, vt, ke + 1, NULL, logits, NULL, NULL);
        pf_set_batch(ctx, batch);
        ctx->lin_log_on = 0;
        if (rc != PINFER_OK) break;
        int a = 0, g = pinfer_argmax(logits, V);
        while (a < ke && vt[a + 1] == g) {
            a++;
            g = pinfer_argmax(logits + (size_t)a * V, V);
        }
        vt[a + 1] = g;
        int e = 0;
        while (e <= a && count < n_max) out[count++] = vt[++e];
        pf_lin_commit(ctx, e);
        ctx->n_past = P + e;
        cur = vt[e];
        if (stats) { stats[1] += ke; stats[2] += a; }
    }
    pf_lin_flush(ctx);
    if (stats) stats[3] += now_ns() - t0;
    free(logits);
    return rc == PINFER_OK || count > 0 ? count : rc;
}

int ref_spec_generate(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt, int32_t *out,
                      int n_max, int k, const int32_t *greedy, uint64_t seed, uint32_t p24,
                      int64_t *stats) {
    return spec_generate(ctx, prompt, n_prompt, out, n_max, k, greedy, seed, p24, stats, 0);
}

int ref_spec_generate_cont(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt, int32_t *out,
                           int n_max, int k, const int32_t *greedy, uint64_t seed, uint32_t p24,
                           int64_t *stats) {
    return spec_generate(ctx, prompt, n_prompt, out, n_max, k, greedy, seed, p24, stats, 1);
}

/* Logits of every row of one forward pass (pf_forward's logits_all) for tests. */
int ref_forward_all(pinfer_ctx *ctx, const int32_t *tokens, int n, float *logits_all) {
    return pf_forward(ctx, tokens, n, NULL, logits_all, NULL);
}
