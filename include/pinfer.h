/* pinfer public C API, B200 build.
 *
 * The same entry points, struct layouts, error codes and ownership rules as the reference
 * engine's engine/include/pinfer.h (version 0.3.0, lines cited per item), so applications and
 * the ctypes bindings (python/pinfer/_lib.py) link against this libpinfer.so unchanged. The
 * implementation runs the forward pass, the speculative verify step, greedy acceptance and
 * the recurrent-state rollback on an NVIDIA B200; host code only validates arguments,
 * uploads the model once and launches work.
 *
 * Every function returns 0 on success or a negative PINFER_E* code unless noted. */
#ifndef PINFER_H
#define PINFER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PINFER_VERSION_MAJOR 0
#define PINFER_VERSION_MINOR 3
#define PINFER_VERSION_PATCH 0

/* error codes (reference pinfer.h:20-27) */
enum {
    PINFER_OK = 0,
    PINFER_E_IO = -1,       /* the model file cannot be opened or read */
    PINFER_E_FORMAT = -2,   /* not a valid .pq file, or a model this build cannot run */
    PINFER_E_NOMEM = -3,    /* host or device allocation failed */
    PINFER_E_ARG = -4,      /* invalid argument */
    PINFER_E_CTX_FULL = -5, /* more tokens than max_ctx */
};

typedef struct pinfer_ctx pinfer_ctx;

/* KV-cache storage formats (reference pinfer.h:34-38). This build stores fp32 rows only;
 * other values are refused with PINFER_E_ARG by pinfer_load. */
enum {
    PINFER_KV_F32 = 0,
    PINFER_KV_F16 = 1,
    PINFER_KV_I8 = 2,
};

/* Load parameters (reference pinfer.h:40-48; same layout). n_threads and gpu_split are
 * accepted for ABI compatibility: the device does the work, and gpu_split must be in [0, 1]. */
typedef struct {
    int n_threads; /* host threads for load-time work; <= 0 means 4 */
    int max_ctx;   /* max tokens kept in the KV cache; <= 0 means 4096 */
    int kv_dtype;  /* PINFER_KV_*; only PINFER_KV_F32 is supported */
    float gpu_split;
} pinfer_params;

pinfer_params pinfer_default_params(void);

/* Load a .pq model onto the current CUDA device (reference pinfer.h:52-53). Returns NULL on
 * failure and stores the error code in *err when err is not NULL. */
pinfer_ctx *pinfer_load(const char *path, const pinfer_params *params, int *err);
void pinfer_free(pinfer_ctx *ctx);

/* Forget all tokens: KV rows, recurrent and conv states (reference pinfer.h:56-57). */
void pinfer_reset(pinfer_ctx *ctx);

/* Feed n tokens in order; logits (may be NULL) receives n_vocab floats for the LAST token
 * (reference pinfer.h:59-60). */
int pinfer_eval(pinfer_ctx *ctx, const int32_t *tokens, int n, float *logits);

/* pinfer_eval, then the last token's logits of ids[0..n_ids) only, bit-identical to the full
 * logits (reference pinfer.h:62-68). */
int pinfer_eval_select(pinfer_ctx *ctx, const int32_t *tokens, int n, const int32_t *ids,
                       int n_ids, float *out);

/* ---- speculative greedy decoding (reference pinfer.h:70-137) ---- */
#define PINFER_SPEC_MAX_K 8

typedef struct {
    int k;
    int draft_vocab;
    int adaptive;
    int ngram;
} pinfer_spec_params;

typedef struct {
    int64_t rounds;
    int64_t drafted;
    int64_t accepted;
    int64_t ngram_rounds;
    int64_t ngram_drafted;
    int64_t ngram_accepted;
} pinfer_spec_stats;

pinfer_spec_params pinfer_default_spec_params(void);

int pinfer_has_mtp(const pinfer_ctx *ctx);

int pinfer_generate_greedy(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt,
                           int32_t *out, int n_max, const pinfer_spec_params *sp,
                           pinfer_spec_stats *stats);

typedef struct {
    const int32_t *stop_ids;
    int n_stop;
    int (*on_token)(int32_t tok, void *user);
    void *user;
} pinfer_gen_opts;

int pinfer_generate_greedy_ex(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt,
                              int32_t *out, int n_max, const pinfer_spec_params *sp,
                              const pinfer_gen_opts *opts, pinfer_spec_stats *stats,
                              int *status);

/* ---- conversation state (reference pinfer.h:139-175) ---- */
size_t pinfer_state_size(const pinfer_ctx *ctx);
int pinfer_state_save(const pinfer_ctx *ctx, void *buf, size_t cap);
int pinfer_state_load(pinfer_ctx *ctx, const void *buf, size_t len);

int pinfer_checkpoint(pinfer_ctx *ctx);
int pinfer_rewind(pinfer_ctx *ctx);
void pinfer_checkpoint_clear(pinfer_ctx *ctx);
int pinfer_checkpoint_n_past(const pinfer_ctx *ctx);

int pinfer_generate_greedy_cont(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt,
                                int32_t *out, int n_max, const pinfer_spec_params *sp,
                                const pinfer_gen_opts *opts, pinfer_spec_stats *stats,
                                int *status);

int pinfer_n_vocab(const pinfer_ctx *ctx);
int pinfer_n_past(const pinfer_ctx *ctx);
int pinfer_eos_id(const pinfer_ctx *ctx);
int pinfer_argmax(const float *logits, int n);
const char *pinfer_version(void);

#ifdef __cplusplus
}
#endif
#endif
