/* B200 extensions of the pinfer C API and the kernel-level C ABI of the verify path.
 *
 * Everything here is additive to include/pinfer.h (the reference grew its own API the same way,
 * engine/include/pinfer.h:62-66,153-155). Device pointers are plain `void *` / typed pointers
 * into CUDA device memory of the current device; `stream` is a cudaStream_t passed as void *
 * (NULL = the legacy default stream). No function here allocates on the CPU side of the model
 * path, and none has a CPU fallback: without a CUDA device they return PINFER_E_NOMEM. */
#ifndef NB_B200_H
#define NB_B200_H

#include <stddef.h>
#include <stdint.h>

#include "pinfer.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the last failure on this thread ("" if none). */
const char *pinfer_b200_last_error(void);

/* Greedy speculative decoding with the benchmark's synthetic drafter (no reference
 * counterpart: the reference drafts with its MTP head, engine/src/spec.c:301-321; this replaces
 * step 1 of pf_spec_decode and keeps steps 2-3, verify / accept / commit, spec.c:323-351).
 * Draft for output index j: with probability p the token greedy[j] (the target's own greedy
 * output, n_max entries, from a plain run), else a uniform token; the drafter is the pure
 * function of (seed, j) in oracle/ref_spec.c. The whole round runs on the device. Resets the
 * context first, like pinfer_generate_greedy_ex. Returns tokens written (out[0..ret)) or a
 * negative PINFER_E_*; *status as in pinfer_generate_greedy_ex; stats accumulated. */
int pinfer_b200_generate_synthetic(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt,
                                   int32_t *out, int n_max, int k, const int32_t *greedy,
                                   uint64_t seed, float p, pinfer_spec_stats *stats, int *status);

/* pinfer_b200_generate_synthetic with append (1: continue after the tokens already in context,
 * like pinfer_generate_greedy_cont) and *decode_ms (may be NULL): device time of the
 * verify / accept loop after the prompt, from CUDA events on the context's stream. */
int pinfer_b200_generate_synthetic_ex(pinfer_ctx *ctx, const int32_t *prompt, int n_prompt,
                                      int32_t *out, int n_max, int k, const int32_t *greedy,
                                      uint64_t seed, float p, int append,
                                      pinfer_spec_stats *stats, int *status, float *decode_ms);

/* Kernel launches in one verify round of draft depth k (the nodes of its CUDA graph). */
int pinfer_b200_round_kernels(pinfer_ctx *ctx, int k);

/* Feed n tokens and return the logits of EVERY row, [n][n_vocab] (the logits_all output of
 * the reference's pf_forward, engine/src/forward.h:293-300). */
int pinfer_b200_forward_all(pinfer_ctx *ctx, const int32_t *tokens, int n, float *logits_all);

/* The CUDA stream every call on ctx runs on (for timing with events on the same stream). */
void *pinfer_b200_stream(pinfer_ctx *ctx);

/* A second context on the same model and device (no reference counterpart): it shares the
 * source's weights in device memory (refcounted; either may be freed first) and owns its own
 * recurrent/conv states, KV cache (max_ctx positions, at most the source's; 0 = the source's),
 * stream and round graphs, so independent request streams can run concurrently, one host thread
 * per context. NULL on failure with *err set. */
pinfer_ctx *pinfer_b200_clone(const pinfer_ctx *src, int max_ctx, int *err);

/* ---- vocab-sharded LM head (the 2B benchmark config) ------------------------------------------
 * No reference counterpart (the reference runs on one device). One context per GPU, each with
 * the same model and fed the same tokens: every GPU runs the layers, and its LM head covers only
 * vocabulary rows [rank * V / world, (rank + 1) * V / world); the greedy argmax of each verify
 * row is merged with one NCCL all-reduce (max) of 64-bit (order-preserving value, first index)
 * keys, so every rank accepts the same tokens, and pinfer_eval's logits are all-gathered.
 * libnccl.so.2 is loaded on first use.
 * pinfer_b200_nccl_id: a 128-byte NCCL unique id, made on one rank and sent to the others by the
 * caller. pinfer_b200_shard_head: collective over the `world` ranks (each calls it with the same
 * id); requires V % (32 * world) == 0; world == 1 undoes sharding. 0, -4 (arguments), -3 (NCCL
 * or CUDA failure, message in pinfer_b200_last_error). */
int pinfer_b200_nccl_id(void *id);
int pinfer_b200_shard_head(pinfer_ctx *ctx, int rank, int world, const void *id);
/* The 64-bit argmax key of (logit v, vocabulary row) the device uses (host function, for
 * checks): unsigned maximum over any partition of the rows = the pf_argmax of all of them. */
unsigned long long nb_argmax_key(float v, int row);

/* ---- multi-sequence batches (no counterpart in the reference, which serves one sequence per
 * context) ---------------------------------------------------------------------------------
 * `slots` (1..2048) sequence slots on a loaded context's weights (shared; the context must outlive the
 * batch), each with its own DeltaNet / conv states, logs and KV cache of max_ctx positions
 * (max_ctx <= the context's), for speculative generation with up to max_k drafts per round.
 * A generation call runs all its sequences in the same passes: the projections of all their
 * rows are one tcgen05 tensor-core GEMM per matrix. NULL on failure (*err set). */
typedef struct pinfer_b200_batch pinfer_b200_batch;
pinfer_b200_batch *pinfer_b200_batch_create(pinfer_ctx *ctx, int slots, int max_ctx, int max_k, int *err);
void pinfer_b200_batch_free(pinfer_b200_batch *b);
/* The CUDA stream (cudaStream_t) the batch's work runs on, for timing with events. */
void *pinfer_b200_batch_stream(pinfer_b200_batch *b);
/* Verify rounds (passes over all the batch's sequences) the last generation ran. */
int pinfer_b200_batch_rounds(const pinfer_b200_batch *b);
/* Greedy speculative generation of n_seq (<= slots) independent sequences from fresh states,
 * with the synthetic drafter of pinfer_b200_generate_synthetic per sequence: prompts
 * concatenated (sequence i has prompt_lens[i] tokens), greedy [n_seq][n_max] and seeds [n_seq]
 * (k > 0), p. k = 0: plain greedy (greedy and seeds may be NULL). Sequence i's tokens go to
 * out[i * n_max ..], their count to counts[i], its generation status to status[i] (may be
 * NULL); the rounds / drafted / accepted counts of all sequences are added to stats (may be
 * NULL); decode_ms (may be NULL): device time of the verify rounds. Every sequence's tokens and
 * counts equal pinfer_b200_generate_synthetic's on its own. 0 or a PINFER_E_* code. */
int pinfer_b200_batch_generate_synthetic(pinfer_b200_batch *b, int n_seq, const int32_t *prompts,
                                         const int32_t *prompt_lens, int n_max, int k, const int32_t *greedy,
                                         const uint64_t *seeds, float p, int32_t *out, int32_t *counts,
                                         int32_t *status, pinfer_spec_stats *stats, float *decode_ms);

/* ---- kernel-level ABI: the Q4K x A8 matmul on device buffers ----------------------------
 * The pf_matmul contract for dtype Q4K_G32 (engine/src/ops.h:49-52: Y[n][rows] = W X, weights
 * read once for all n) with the reference's arithmetic (kern_quant_act, kern_act.c:14-41;
 * kern_q4k, kern_quant.c:296-304): bit-identical outputs. Weights are in the panel layout
 * (nb_q4k_repack of the .pq bytes, then copied to the device). */
size_t nb_q4k_panel_bytes(int rows, int cols);
/* .pq Q4K tiles (host) -> panel layout (host), panel_bytes(rows, cols) bytes. 0 or -4. */
int nb_q4k_repack(const uint8_t *pq, int rows, int cols, uint8_t *panels);

typedef struct nb_mv nb_mv;
/* Activation scratch (A8 of up to nmax vectors of `cols`) and a control block on the device.
 * nmax <= NB_MV_MAX_N. NULL on failure (no device, bad shape). Calls with n <= 16 vectors run
 * the CUDA-core matvec kernels; n > 16 (which needs nmax > 16 at creation) runs the tcgen05
 * tensor-core GEMM, with bit-identical results. */
#define NB_MV_MAX_N 65536
nb_mv *nb_mv_create(int rows, int cols, int nmax);
void nb_mv_destroy(nb_mv *h);
/* Set the vector count n (1..nmax) used by the next calls (one tiny kernel on `stream`). */
int nb_mv_set_n(nb_mv *h, int n, void *stream);
/* A8-quantise X [n][cols] (device fp32) into the scratch: kern_quant_act. */
int nb_mv_quant(nb_mv *h, const float *X, void *stream);
/* Y [n][rows] = W (device panel layout) x scratch activations. */
int nb_mv_matmul(nb_mv *h, const void *W, float *Y, void *stream);
/* `iters` back-to-back nb_mv_matmul launches, launch i reading weights at W + (i % copies) *
 * stride (a rotating arena of copies, so timed launches stream from HBM). For timing. */
int nb_mv_matmul_repeat(nb_mv *h, const void *W, size_t stride, int copies, float *Y, int iters,
                        void *stream);
/* The same with the LM-head kernel (logits into Y, may be NULL; argmax keys into partial
 * [n][rows/32] uint64, NaN flags into nan0 [n]). */
int nb_mv_head_repeat(nb_mv *h, const void *W, size_t stride, int copies, float *Y, int iters,
                      void *partial, int *nan0, void *stream);
/* Tensor-core path, two steps. nb_mv_prepare widens W0 (rows x cols, panel layout), or the row
 * concatenation W0 ++ W1 when W1 is not NULL (gate / up, rows % 32 == 0), into the handle's
 * tile image (the int8 codes in the tensor cores' shared-memory layout plus the scale entries;
 * needs nmax > 16). nb_mv_gemm then runs on the current n (> 16) vectors:
 * epi 0: Y [n][rows] = W0 x;  1: Y += W0 x (residual add);
 * 3 (prepared with W1): A8 of silu(W0 x) * (W1 x) into q [n][rows] int8, d / fs [n][rows / 32]
 *    (pf_silu_mul then kern_quant_act);
 * 4: LM head: logits into Y (may be NULL), argmax keys into partial [n][rows / 32] uint64 and
 *    row-0 NaN flags into nan0 [n], as nb_mv_head_repeat.
 * nb_mv_matmul with n > 16 is nb_mv_prepare(W) + nb_mv_gemm(0). 0, or -4 (arguments). */
int nb_mv_prepare(nb_mv *h, const void *W0, const void *W1, void *stream);
int nb_mv_gemm(nb_mv *h, int epi, float *Y, void *q, void *d, void *fs, void *partial, int *nan0,
               void *stream);
/* The status word of the tensor-core path (0, or -91 after a bounded device wait gave up);
 * synchronous. */
int nb_mv_status(nb_mv *h);
/* nb_mv_quant + nb_mv_matmul. */
int nb_mv_run(nb_mv *h, const void *W, const float *X, float *Y, void *stream);
/* Copy the scratch activations out (device buffers: q [n][cols] int8, d / fsum [n][cols/32]). */
int nb_mv_get_act(nb_mv *h, int8_t *q, float *d, float *fsum, void *stream);

/* Test hooks for the glibc expf / log1pf restatement the DeltaNet gates use
 * (engine/src/forward_lin.c:19,290-293 call the C library's expf and log1pf).
 * nb_libm_selftest: the restatement compiled for the host against the C library on every
 * `stride`-th 32-bit input (stride 1 = all 2^32), `threads` host threads; mismatch count in
 * *mismatches; 0 or -1. nb_libm_eval_host: the C library's values (fn 0 expf, 1 log1pf) of host
 * arrays. nb_libm_eval_device: the device restatement on device arrays, on `stream`. */
int nb_libm_selftest(int threads, long long stride, long long *mismatches);
int nb_libm_eval_host(int fn, const float *x, float *y, long long n);
int nb_libm_eval_device(int fn, const float *x, float *y, long long n, void *stream);

/* Test hook of the bounded device waits: a one-warp kernel waits on an mbarrier whose expected
 * bytes never arrive, gives up after spin_limit polls (1 .. 2^22), records -90 in a status word
 * and returns; *status_out receives that word. 0, -4 (arguments), -3 (CUDA error). */
int nb_test_bounded_wait(unsigned spin_limit, int *status_out);

/* Host test hooks of the state blob's narrow K / V rows (pinfer_params.kv_dtype; the reference's
 * format, engine/src/state.c:64-83 with forward_kv.c:83-123): nb_test_kv_f16 dir 0 writes the
 * binary16 bits of n floats that binary16 represents exactly (NaN: quiet, top payload bits),
 * dir 1 the floats of n binary16 bit patterns; nb_test_kv_i8 the int8 codes of rows of widened
 * values q * scale (one scale per row of hd). 0, or -4 (arguments). No device needed. */
int nb_test_kv_f16(int dir, const void *in, void *out, long long n);
int nb_test_kv_i8(const float *v, const float *scales, int rows, int hd, int8_t *q);

/* Allocation-free Q4K x A8 matmul. No counterpart in the reference (its CPU pf_matmul takes
 * caller buffers and needs no scratch).
 * Y [n][rows] = W (device panel layout) x A8(X [n][cols]), the same kernels and the same
 * bit-exact result as nb_mv_create(rows, cols, n) + nb_mv_set_n + nb_mv_run, but the scratch
 * (A8 activations and the control block) lives in a fixed array inside the library's device
 * image, so the call performs no cudaMalloc / cudaFree and calls no allocating library routine.
 * Meant for hosts that must not allocate device memory while they call it (their own allocator
 * holds the device's memory, or they cannot take an allocation's device-wide sync).
 * Limits: n <= NB_MV_STATIC_MAX_N, cols <= NB_MV_STATIC_MAX_COLS; larger sizes return -4 and
 * set pinfer_b200_last_error. The first call on each device does setup (looks up the scratch's
 * device address with that device current and sets the kernels' shared-memory limits) and
 * should come before any stream capture. One scratch per device: calls that overlap in time on
 * one device (other streams or threads) race on it and must be serialised by the caller.
 * The call returns once Y is written (it waits for `stream`), after reading the status word of
 * the kernels' bounded device waits: -3 with pinfer_b200_last_error set if one gave up.
 * The scratch takes NB_MV_STATIC_BYTES of every device that loads the library, until exit.
 * 0, -4 (arguments), -3 (CUDA error or a device wait that gave up). */
#define NB_MV_STATIC_MAX_N 16
#define NB_MV_STATIC_MAX_COLS 8192
#define NB_MV_STATIC_STEP_BYTES 768       /* the control block, padded to 256 B */
#define NB_MV_STATIC_BYTES 164608         /* 768 + 16 x 8192 + 2 x 16 x 256 x 4 */
int nb_mv_run_static(const void *W, int rows, int cols, const float *X, int n, float *Y,
                     void *stream);

#ifdef __cplusplus
}
#endif
#endif
