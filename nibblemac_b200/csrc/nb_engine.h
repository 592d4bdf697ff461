// Internal interface between the host engine (nb_engine.cu, C++) and the device kernels
// (nb_kernels.cu). Not part of the public API.
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda.h>
#include <cuda_runtime.h>

#include "nb_math.cuh"
#include "pinfer.h"

namespace nb {

// ---- Q4K weights in HBM: the panel layout -------------------------------------------------
// The .pq file stores Q4K_G32 as 4-row tiles of 576-byte superblocks (engine/FORMAT.md,
// "Quantized dtypes"). At upload every matrix is repacked, without touching a code or a
// scale value, into panels of 32 rows: for panel p and superblock sb (256 columns) one
// 4608-byte unit holds
//   [32 rows x 16 B scale entry][block 0: 32 rows x 16 B codes] ... [block 7: 32 x 16 B]
// so a warp with lane = row reads every part of the unit with one coalesced 512-byte load.
// Scale entry of a row (two little-endian u64): A = s6[0..7] (6 bits each, bits 6k..6k+5) |
// D fp16 bits << 48, B = m6[0..7] | M fp16 bits << 48. Codes: byte j holds column j (low
// nibble) and column j + 16 (high nibble) of the 32-column block, as in the file.
constexpr int kPanelRows = 32;
constexpr int kUnitBytes = 4608;

struct Mat {
    const uint8_t *w = nullptr;  // panel layout
    int rows = 0, cols = 0, npanels = 0, nsb = 0;
};

// int8 activations, vector-major: q [nmax][cols], d / fs [nmax][cols / 32]
struct Act {
    int8_t *q = nullptr;
    float *d = nullptr, *fs = nullptr;
    int cols = 0;
};

constexpr int kMaxRows = 16;      // rows (tokens) per forward pass on the small-batch path
constexpr int kMaxLayers = 32;

// Mutable per-pass control block in device memory. Kernels read the pass shape from it, so a
// captured CUDA graph replays a whole verify round with no host round trip.
struct Step {
    int n;                 // rows in this pass (0 = nothing to do)
    int pos0;              // position of row 0 (= tokens already in context)
    int logged;            // 1: verify pass (rows >= 1 on state copies, logged for commit)
    int wr;                // log half the next logged pass writes
    int pend_keep;         // recurrent updates (log rows 1..pend_keep of half wr^1) to replay
    int pend_conv;         // conv commit owed: keep = pend_conv tokens of the last logged pass
    int row0;              // first row of this sequence's rows in a multi-sequence pass (else 0)
    int tokens[kMaxRows];  // input tokens of the pass
    int argmax[kMaxRows];  // head argmax of every row (first maximum)
    // generation loop (nb_accept)
    int count, n_max, done, status;
    int k;                 // drafts per round
    int eos;               // stop token (< 0: none)
    int n_stop;
    int stop_ids[8];
    int cur;
    int max_ctx;
    int vocab;
    unsigned p24;          // synthetic drafter acceptance threshold (p * 2^24)
    unsigned long long seed;
    long long rounds, drafted, accepted;
    // MTP drafting (drafter 1): the last MTP pass's draft and the last verify's committed rows
    int drafter;           // 0 synthetic (seed, p24, greedy stream), 1 the MTP head
    int mtp_d1;
    int last_pos, last_e;
    int last_tok[kMaxRows];
    // prompt lookup (n-gram drafts, engine/src/ngram.c): the history of fed and emitted tokens
    // and its hash index, on the device
    int ngram;             // longest n-gram draft (0: none)
    int use_ng;            // the coming round drafts from the history
    int hist_n, hist_idx;  // tokens in the history; n-grams ending before hist_idx are indexed
    int hist_cap, ng_bits;
    int *hist, *ng_tab;    // [hist_cap], [3][1 << ng_bits]: end position + 1, 0 = empty
    long long ng_rounds, ng_drafted, ng_accepted;
    // adaptive speculation (engine/src/spec_adapt.c): the chain runs on while the newest
    // draft's top-1 probability is high enough; plain steps while speculation measures slower
    int adaptive;
    int chain_stop;                   // this round's chain stopped early
    int last_n;                       // rows of the round just committed
    float conf;                       // top-1 probability of the newest MTP draft
    unsigned long long t_stamp[3];    // %globaltimer: round start, verify start, verify end
    double ad_tv[kMaxRows + 1];       // EMA seconds of a verify pass of n rows
    double ad_t_plain, ad_r_tok, ad_r_sec;
    int ad_n_spec, ad_plain_mode, ad_plain_run, ad_probe_after, ad_probing;
};

struct GenArgs {
    int n_max, k, eos, n_stop, max_ctx, vocab, drafter, ngram, adaptive;
    int stop_ids[8];
    unsigned p24;
    unsigned long long seed;
};

// Per-layer parameters of a Gated DeltaNet layer on the device
struct LinLayer {
    float *conv_state;     // [K-1][C]
    float *rec;            // [nv][dk][dv]
    float *xin;            // [cap][C] raw conv inputs of rows 1.. of a logged pass
    float *upd;            // [2][cap][nv][dk + dv + 1]
    const float *conv_w;   // [C][K]
    const float *A;        // [nv] = -expf(A_log) (computed on the host with glibc) or A
    const float *dt_bias;  // [nv]
    const float *norm_w;   // [dv]
};

struct LinDims {
    int C, K, kd, vd, nk, nv, rep, dk, dv, cap, ldy;
    float eps;
    // per-sequence strides (floats) of a multi-sequence batch's states; 0 for one context
    size_t ss_conv = 0, ss_rec = 0, ss_xin = 0, ss_upd = 0;
};

struct AttnLayer {
    float *kc, *vc;        // [nkv][max_ctx][hd], fp32 (with fp16 / int8 storage: the widened values)
    const float *q_norm, *k_norm;
    float *ks = nullptr, *vs = nullptr;   // int8 storage: row scales [nkv][max_ctx] (for the state blob)
};

struct AttnDims {
    int nq, nkv, hd, rot, max_ctx, ldy;
    float eps;
    const float *rope_cos, *rope_sin;   // [max_ctx][rot / 2]
    int rps = kMaxRows;                 // rows per sequence in the launch grid
    int kv_dtype = 0;                   // PINFER_KV_*: the precision K / V rows are stored at
    size_t ss_kv = 0;                   // per-sequence stride (floats) of a batch's KV caches
};

// ---- launchers (nb_kernels.cu); all asynchronous on `s` ---------------------------------
// Multi-sequence passes: `nseq` Step blocks (st[0..nseq)), sequence i's rows at st[i].row0 ..;
// `rps` = the most rows any sequence has in the pass.
void launch_embed(const Mat &E, const Step *st, float *x, int H, cudaStream_t s, int nseq = 1, int rps = kMaxRows);
void launch_norm_quant(const float *x, const float *w, int H, float eps, const Step *st,
                       Act out, cudaStream_t s, int nseq = 1, int rps = kMaxRows);
// Y = W A8(x): mode 0 store y[v][ldy], mode 1 residual x[v][ldy] += y
void launch_matvec(const Mat &W, Act in, const Step *st, float *y, int ldy, int mode, int nmax,
                   cudaStream_t s);
void launch_matvec_chunked(const Mat &W, Act in, const Step *st, float *y, int ldy, int mode,
                           int nmax, cudaStream_t s);
// Byte ranges (16-byte aligned, sizes multiples of 16) a kernel asks the L2 to fetch ahead of
// the kernels that will read them (cp.async.bulk.prefetch.L2), split over the kernel's CTAs.
// A range with row_bytes > 0 is a KV cache: only its first (Step::pos0 + Step::n) rows of
// row_bytes are fetched (the positions the pass attends to), read from the Step block when the
// kernel starts.
constexpr int kMaxPrefetch = 12;
struct L2Prefetch {
    const void *p[kMaxPrefetch] = {};
    unsigned bytes[kMaxPrefetch] = {};
    unsigned row_bytes[kMaxPrefetch] = {};
    int n = 0;
    void add(const void *ptr, size_t nbytes, unsigned rowb = 0) {
        if (n < kMaxPrefetch && ptr && nbytes >= 16) {
            p[n] = ptr;
            bytes[n] = (unsigned)(nbytes & ~(size_t)15);
            row_bytes[n] = rowb;
            n++;
        }
    }
};
// The same with the RMSNorm + A8 of the residual rows x fused into the kernel (scratch: the A8
// buffer a fallback path may use for large passes); pf: ranges to prefetch into L2
void launch_matvec_norm(const Mat &W, const float *x, const float *w, float eps, const Step *st,
                        float *y, int ldy, int nmax, Act scratch, cudaStream_t s,
                        const L2Prefetch &pf = L2Prefetch());
void launch_matvec_swiglu_norm(const Mat &G, const Mat &U, const float *x, const float *w, float eps,
                               const Step *st, Act out, int nmax, Act scratch, cudaStream_t s);
// With fbest / fctr (nmax <= 4, one context, unsharded) the kernel also finishes the argmax into
// Step::argmax (no launch_argmax_final): fbest [4][grid] keys, fctr a zeroed counter it resets.
constexpr int kHeadFuseSlots = 4 * 1024;
void launch_matvec_head_norm(const Mat &W, const float *x, const float *w, float eps, const Step *st,
                             float *logits, int ld, unsigned long long *partial, int *nan0, int nmax,
                             cudaStream_t s, int row_base = 0, unsigned long long *fbest = nullptr,
                             int *fctr = nullptr);
// gate / up with SwiGLU and A8 quantisation of the product
void launch_matvec_swiglu(const Mat &G, const Mat &U, Act in, const Step *st, Act out, int nmax,
                          cudaStream_t s);
// tied head: logits (may be null) [v][ld] and per-panel argmax partials; row_base is the
// vocabulary index of W's row 0 (a vocab shard), which the argmax keys carry
void launch_matvec_head(const Mat &W, Act in, const Step *st, float *logits, int ld,
                        unsigned long long *partial, int *nan0, int nmax, cudaStream_t s, int row_base = 0);
void launch_argmax_final(const unsigned long long *partial, const int *nan0, int npanels,
                         Step *st, cudaStream_t s, int nseq = 1, int rps = kMaxRows);
// vocab-sharded head: per-row best keys and NaN flags into keys [2][kMaxRows] (to be merged by
// an all-reduce max across the shards), then the merged keys into Step::argmax
void launch_argmax_keys(const unsigned long long *partial, const int *nan0, int npanels, const Step *st,
                        unsigned long long *keys, cudaStream_t s, int kstride = kMaxRows, int nseq = 1,
                        int rps = kMaxRows);
void launch_keys_argmax(const unsigned long long *keys, Step *st, cudaStream_t s, int kstride = kMaxRows,
                        int nseq = 1, int rps = kMaxRows);
// nseq > 1 needs the fast kernel's shape (deltanet_batch_ok); keep_max: the most deferred
// updates a pass may replay (a context: PINFER_SPEC_MAX_K; a batch: its draft depth)
void launch_deltanet(const LinLayer &L, const LinDims &d, const float *y,
                     Step *st, Act out, cudaStream_t s, int nseq = 1, int rps = kMaxRows,
                     int keep_max = PINFER_SPEC_MAX_K);
bool deltanet_batch_ok(const LinDims &d);
// a prefill chunk's rows 0..n-1 of y (no deferred commit, nothing logged; the shape
// deltanet_batch_ok accepts): prep, recurrence and post kernels through two scratch buffers,
// recs (deltanet_rec_floats) and o_rows ([n][vd])
size_t deltanet_rec_floats(const LinDims &d, int rows);
void launch_deltanet_rows(const LinLayer &L, const LinDims &d, const float *y, int n, float *recs, float *o_rows,
                          Act out, int *status, cudaStream_t s);
// the same for an unlogged pass of up to 16 rows per sequence of a batch (R rows in all;
// sequence i's rows at st[i].row0, its states at d's per-sequence strides)
void launch_deltanet_rows_seqs(const LinLayer &L, const LinDims &d, const float *y, int R, Step *st, int nseq,
                               float *recs, float *o_rows, Act out, cudaStream_t s);
// attention grids cover d.rps rows of each of nseq sequences; nseq > 1 needs the cluster kernel
// (attn_batch_ok)
void launch_attn_prep(const AttnLayer &L, const AttnDims &d, const float *y, float *qbuf,
                      const Step *st, cudaStream_t s, int nseq = 1);
void launch_attn(const AttnLayer &L, const AttnDims &d, const float *y, const float *qbuf,
                 const Step *st, Act out, cudaStream_t s, int nseq = 1);
bool attn_batch_ok(const AttnDims &d);
// the sub-passes of one context's prefill chunk (nseq Step blocks over one KV cache): one CTA per
// (row, KV group) with the group's query heads, else as launch_attn
void launch_attn_rows(const AttnLayer &L, const AttnDims &d, const float *y, const float *qbuf, const Step *st,
                      Act out, cudaStream_t s, int nseq);
// greedy / out: sequence i's at greedy + i * n_max, out + i * n_max
void launch_gen_start(Step *st, const int *greedy, int *out, cudaStream_t s, int nseq = 1);
void launch_accept(Step *st, const int *greedy, int *out, cudaStream_t s, int nseq = 1);
void launch_pass_end(Step *st, cudaStream_t s, int nseq = 1);
// MTP draft head (see the kernels' comments)
void launch_norm_rows(const float *x, const float *w, int H, float eps, const Step *st, float *out,
                      cudaStream_t s, int nseq = 1);
void launch_mtp_input(const Mat &E, const float *h, const Step *ms, const float *w_emb, const float *w_hid,
                      int H, float eps, Act out, cudaStream_t s, int nseq = 1);
void launch_mtp_chain_set(Step *st, Step *ms, int step, cudaStream_t s);
void launch_mtp_chain_take(Step *st, const Step *ms, int step, const float *mrows, float *mcur, int H,
                           cudaStream_t s);
void launch_mtp_pending_set(const Step *st, Step *ms, cudaStream_t s);
void launch_mtp_pending_take(Step *st, const Step *ms, const float *mrows, float *mcur, int H, cudaStream_t s);
void launch_mtp_prefill_fix(const Step *st, Step *ms, cudaStream_t s);
// adaptive speculation: a %globaltimer stamp into st->t_stamp[idx]; the top-1 probability of
// the last row of an MTP head pass (logits [rows][ld], draft vocabulary nv) into st->conf
void launch_stamp(Step *st, int idx, cudaStream_t s);
void launch_conf(const float *logits, int ld, int nv, const Step *ms, Step *st, cudaStream_t s);
size_t deltanet_smem(int rep);
void launch_set_pass(Step *st, int n, int pos0, int logged, const int *tokens, cudaStream_t s);
void launch_set_gen(Step *st, const GenArgs &g, cudaStream_t s, int nseq = 1,
                    const unsigned long long *seeds = nullptr);
int kernels_init(int max_ctx, int hd, int rep);
// Records the message pinfer_b200_last_error returns on this thread.
void set_last_error(const char *msg);   // 0, or -1 if a CUDA call failed
void launch_flush(const LinLayer *layers, int n_lin, const LinDims &d, Step *st, cudaStream_t s, int nseq = 1);
// Host-chosen shapes of a multi-sequence pass: per sequence n, pos0, row0, logged, tokens.
struct SeqPass {
    int n, pos0, row0, logged;
    int tokens[kMaxRows];
};
void launch_set_pass_seqs(Step *st, const SeqPass *dev_passes, int nseq, cudaStream_t s);
// count of sequences with Step::done set, into *ndone
void launch_count_done(const Step *st, int nseq, int *ndone, cudaStream_t s);
// small-n standalone entry points for the C-ABI kernel tests
void launch_quant_act(const float *x, int n, int cols, Act out, cudaStream_t s);

// ---- tensor-core GEMM for passes of many rows (nb_gemm.cu) --------------------------------
// TMA descriptors of an A8 activation buffer of `rows` rows (codes, block scales, block sums).
struct GemmMaps {
    CUtensorMap q[3], d[3], fs[3];   // boxes of 16, 32 and 64 rows (the GEMM's activation tile heights)
    int rows = 0, cols = 0;
};
// A matrix (or the row concatenation of two) in the tensor-core tile image: per tile of 128
// rows and superblock of 256 columns, the codes widened to int8 in the MMA's swizzled layout
// and the 4 panels' scale entries (gemm_tiled_bytes; made by launch_gemm_tile).
struct GemmW {
    const uint8_t *t = nullptr;
    int rows = 0, cols = 0, npanels = 0, nsb = 0, mtiles = 0;
};
struct GemmArgs {
    GemmW W;
    int n = 0;                              // activation rows
    float *y = nullptr;                     // epilogue 0 / 1 output, 4: logits (may be null)
    int ldy = 0;
    unsigned long long *partial = nullptr;  // epilogue 4: argmax keys [n][npanels]
    int *nan0 = nullptr;
    int row_base = 0;
    int *status = nullptr;                  // set to -91 when a bounded device wait gives up
};
int gemm_maps(const Act &a, int rows, GemmMaps *m);   // 0 or -1 (message in last error)
int gemm_init();                                       // shared-memory limits; 0 or -1
size_t gemm_tiled_bytes(int rows, int cols);
// the tile image of W0 ++ W1 (W1.npanels = 0: W0 alone; with W1, W0.rows % 32 == 0)
GemmW gemm_w(const Mat &W0, const Mat &W1, uint8_t *tiled);
void launch_gemm_tile(const Mat &W0, const Mat &W1, uint8_t *tiled, cudaStream_t s);
// Y = W A8(x) over g.n rows with the given epilogue (0 store, 1 residual add, 4 head keys); the
// A8 rows come through `maps`
void launch_gemm(int epi, const GemmMaps &maps, const GemmArgs &g, cudaStream_t s);
// A8 of silu(gate) * up, gate = y[v][0, ffn), up = y[v][ffn, 2 ffn)
void launch_swiglu_quant(const float *y, int ldy, int ffn, int n, Act out, cudaStream_t s);

// ---- host-side helpers -----------------------------------------------------------------------
size_t panel_bytes(int rows, int cols);
// repack one Q4K matrix (.pq tile layout, rows % 4 == 0, cols % 256 == 0) into the panel
// layout; `out` has panel_bytes(rows, cols) bytes; rows beyond `rows` are zero.
void repack_q4k(const uint8_t *pq, int rows, int cols, uint8_t *out);


}  // namespace nb
