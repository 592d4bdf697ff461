// Multi-sequence batch engine (pinfer_b200_batch_*): many independent requests on one GPU in
// the same passes, so every weight matrix is read once per pass for all of them and the
// projections become tcgen05 tensor-core GEMMs over the merged rows.
//
// The reference serves one sequence per context (pinfer.h); a server would run one context per
// request. Here S sequence slots share one copy of the weights (the loaded context's, plus the
// tensor cores' tile image made at creation) and keep their own DeltaNet states, conv states,
// logs and KV caches in strided per-sequence arrays. A pass lays the sequences' rows one after
// another (sequence i at Step[i].row0 ..): the row-wise kernels (embedding, RMSNorm + A8,
// SwiGLU) and the GEMMs see one R-row matrix, the DeltaNet and attention kernels take a grid
// dimension per sequence and read that sequence's Step block and states. Every row's
// arithmetic is the single-context path's, so each sequence's tokens are identical to a
// generation on its own (and to the reference's).
//
// Generation: prefill all prompts but their last token in chunks of up to 16 rows per sequence
// (passes of sum-of-chunk rows; sequences drop out as their prompts end), one pass over every
// last prompt token with the LM head (the first generated token), then verify rounds of k + 1
// rows per sequence replayed from one CUDA graph: draft (synthetic drafter), verify, greedy
// acceptance and commit per sequence on the device, with no host round trip until every
// sequence has finished.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

#include "nb_b200.h"
#include "nb_ctx.h"

using namespace nb;

struct pinfer_b200_batch {
    pinfer_ctx *src = nullptr;
    std::shared_ptr<WeightStore> weights;   // keeps the parameters alive with the batch
    int device = 0;
    int S = 0, max_ctx = 0, kmax = 0, rmax = 0;
    cudaStream_t stream = nullptr;
    std::vector<void *> allocs;

    struct Layer {
        GemmW win, out, gu, down;   // tile images (gu: gate ++ up)
    } layers[kMaxLayers];
    GemmW head;
    LinLayer lin[kMaxLayers];
    AttnLayer att[kMaxLayers];
    LinDims lind{};
    AttnDims attd{};

    float *x = nullptr, *y = nullptr, *qbuf = nullptr;
    int ldy = 0;
    Act act_h, act_mid;
    GemmMaps maps_h, maps_ol, maps_oa, maps_f;
    unsigned long long *partial = nullptr;
    int *nan0 = nullptr;
    unsigned long long *keys = nullptr;   // vocab-sharded head: [2][rmax] per-row keys, merged by NCCL
    bool sharded = false;
    int row_base = 0;
    int *status = nullptr;
    float *dn_recs = nullptr, *dn_o = nullptr;   // prefill passes' DeltaNet records and raw outputs
    Step *steps = nullptr, *h_steps = nullptr;
    SeqPass *d_pass = nullptr, *h_pass = nullptr;
    int pass_slots = 0;
    int *d_out = nullptr, *d_greedy = nullptr;
    size_t out_cap = 0;
    unsigned long long *d_seeds = nullptr;
    int *d_ndone = nullptr, *h_ndone = nullptr;

    cudaGraphExec_t graph = nullptr;
    int graph_nseq = -1, graph_k = -1;
    int last_rounds = 0;   // verify rounds (graph replays) of the last generation
    const int *graph_out = nullptr;

    template <class T>
    int dalloc(T **p, size_t bytes) {
        void *q = nullptr;
        if (cudaMalloc(&q, bytes ? bytes : 16) != cudaSuccess) {
            set_last_error("pinfer_b200_batch: device allocation failed");
            return PINFER_E_NOMEM;
        }
        allocs.push_back(q);
        *p = (T *)q;
        return PINFER_OK;
    }
    ~pinfer_b200_batch() {
        if (graph) cudaGraphExecDestroy(graph);
        for (void *p : allocs) cudaFree(p);
        if (h_steps) cudaFreeHost(h_steps);
        if (h_pass) cudaFreeHost(h_pass);
        if (h_ndone) cudaFreeHost(h_ndone);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

int tile_mat(pinfer_b200_batch *b, const Mat &W0, const Mat &W1, GemmW *out) {
    uint8_t *t = nullptr;
    const int rows = W1.npanels ? W0.npanels * kPanelRows + W1.rows : W0.rows;
    int rc = b->dalloc(&t, gemm_tiled_bytes(rows, W0.cols));
    if (rc) return rc;
    launch_gemm_tile(W0, W1, t, b->stream);
    *out = gemm_w(W0, W1, t);
    return PINFER_OK;
}

void gemm(pinfer_b200_batch *b, int epi, const GemmMaps &maps, const GemmW &W, int R, float *y, int ldy) {
    GemmArgs g;
    g.W = W;
    g.n = R;
    g.y = y;
    g.ldy = ldy;
    g.partial = b->partial;
    g.nan0 = b->nan0;
    g.row_base = epi == 4 ? b->row_base : 0;
    g.status = b->status;
    launch_gemm(epi, maps, g, b->stream);
}

Act with_cols(Act a, int cols) {
    a.cols = cols;
    return a;
}

// One pass over R rows of nseq sequences (at most rps rows each), the shapes in the Step blocks.
// prefill: an unlogged pass with no deferred commit (the prompts' passes), whose DeltaNet layers
// run as conv / norms in parallel, the recurrence with its state in registers, the gated norms.
void enqueue_forward(pinfer_b200_batch *b, int R, int nseq, int rps, bool head, bool prefill = false) {
    const pinfer_ctx *c = b->src;
    cudaStream_t s = b->stream;
    launch_embed(c->embed, b->steps, b->x, c->H, s, nseq, rps);
    AttnDims ad = b->attd;
    ad.rps = rps;
    for (int l = 0; l < c->n_layers; l++) {
        const auto &D = c->layers[l];
        const auto &T = b->layers[l];
        launch_norm_quant(b->x, D.in_norm, c->H, c->eps, b->steps, b->act_h, s, nseq, rps);
        if (D.is_full) {
            gemm(b, 0, b->maps_h, T.win, R, b->y, c->attd.ldy);
            const Act o = with_cols(b->act_mid, c->nq * c->hd);
            launch_attn_prep(b->att[l], ad, b->y, b->qbuf, b->steps, s, nseq);
            launch_attn(b->att[l], ad, b->y, b->qbuf, b->steps, o, s, nseq);
            gemm(b, 1, b->maps_oa, T.out, R, b->x, c->H);
        } else {
            gemm(b, 0, b->maps_h, T.win, R, b->y, c->lind.ldy);
            const Act o = with_cols(b->act_mid, c->vd);
            if (prefill)
                launch_deltanet_rows_seqs(b->lin[D.lin], b->lind, b->y, R, b->steps, nseq, b->dn_recs, b->dn_o, o, s);
            else
                launch_deltanet(b->lin[D.lin], b->lind, b->y, b->steps, o, s, nseq, rps, b->kmax);
            gemm(b, 1, b->maps_ol, T.out, R, b->x, c->H);
        }
        launch_norm_quant(b->x, D.post_norm, c->H, c->eps, b->steps, b->act_h, s, nseq, rps);
        gemm(b, 0, b->maps_h, T.gu, R, b->y, 2 * c->ffn);
        launch_swiglu_quant(b->y, 2 * c->ffn, c->ffn, R, with_cols(b->act_mid, c->ffn), s);
        gemm(b, 1, b->maps_f, T.down, R, b->x, c->H);
    }
    if (head) {
        launch_norm_quant(b->x, c->norm, c->H, c->eps, b->steps, b->act_h, s, nseq, rps);
        gemm(b, 4, b->maps_h, b->head, R, nullptr, 0);
        if (!b->sharded) {
            launch_argmax_final(b->partial, b->nan0, b->head.npanels, b->steps, s, nseq, rps);
        } else {
            // this GPU's vocabulary rows only: per-row best keys (global row indices), one
            // all-reduce (max) across the shards, then tokens exactly as the unsharded path
            launch_argmax_keys(b->partial, b->nan0, b->head.npanels, b->steps, b->keys, s, b->rmax, nseq, rps);
            nccl_api(nullptr, 0)->all_reduce(b->keys, b->keys, 2 * (size_t)b->rmax, ncclUint64, ncclMax,
                                             c->nccl, s);
            launch_keys_argmax(b->keys, b->steps, s, b->rmax, nseq, rps);
        }
    }
    launch_pass_end(b->steps, s, nseq);
}

int batch_alloc(pinfer_b200_batch *b) {
    const pinfer_ctx *c = b->src;
    const int S = b->S;
    int rc;
    NB_CUDA_OK(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    if (kernels_init(b->max_ctx, c->hd, c->lind.rep) != 0) {
        set_last_error("pinfer_b200_batch_create: kernel setup failed");
        return PINFER_E_NOMEM;
    }
    // tile images of every projection (shared with the context's prefill and its clones) and
    // of this batch's head rows
    if ((rc = ensure_gemm_tiles(b->src, false))) return rc;
    for (int l = 0; l < c->n_layers; l++) {
        const auto &W = b->weights->tiles[l];
        b->layers[l] = {W.win, W.out, W.gu, W.down};
    }
    b->sharded = c->shard_world > 1;
    b->row_base = b->sharded ? c->head_row0 : 0;
    if ((rc = tile_mat(b, b->sharded ? c->head_view : c->head, Mat(), &b->head))) return rc;

    // per-sequence states, strided by sequence
    const int cap = b->kmax + 1;
    b->lind = c->lind;
    b->lind.cap = cap;
    b->lind.ss_conv = (size_t)std::max(c->K - 1, 1) * c->C;
    b->lind.ss_rec = (size_t)c->nv * c->dk * c->dv;
    b->lind.ss_xin = (size_t)cap * c->C;
    b->lind.ss_upd = (size_t)2 * cap * c->nv * (c->dk + c->dv + 1);
    b->attd = c->attd;
    b->attd.max_ctx = b->max_ctx;
    b->attd.ss_kv = (size_t)c->nkv * b->max_ctx * c->hd;
    if (!deltanet_batch_ok(b->lind) || !attn_batch_ok(b->attd)) {
        set_last_error("pinfer_b200_batch_create: this model shape has no multi-sequence kernels");
        return PINFER_E_FORMAT;
    }
    for (int l = 0; l < c->n_layers; l++) {
        const auto &D = c->layers[l];
        if (D.is_full) {
            AttnLayer &A = b->att[l];
            A = c->att[l];
            A.ks = A.vs = nullptr;   // int8 row scales serve the context's state blob only
            const size_t kv = sizeof(float) * S * b->attd.ss_kv;
            if ((rc = b->dalloc(&A.kc, kv)) || (rc = b->dalloc(&A.vc, kv))) return rc;
        } else {
            LinLayer &N = b->lin[D.lin];
            N = c->lin[D.lin];
            if ((rc = b->dalloc(&N.conv_state, sizeof(float) * S * b->lind.ss_conv)) ||
                (rc = b->dalloc(&N.rec, sizeof(float) * S * b->lind.ss_rec)) ||
                (rc = b->dalloc(&N.xin, sizeof(float) * S * b->lind.ss_xin)) ||
                (rc = b->dalloc(&N.upd, sizeof(float) * S * b->lind.ss_upd)))
                return rc;
        }
    }
    // activations of the largest pass (prefill: kMaxRows rows per sequence)
    const size_t R = (size_t)S * kMaxRows;
    b->rmax = (int)R;
    b->ldy = std::max(std::max(c->lind.ldy, c->attd.ldy), 2 * c->ffn);
    const int mid = std::max(std::max(c->vd, c->nq * c->hd), c->ffn);
    if ((rc = b->dalloc(&b->x, sizeof(float) * R * c->H)) || (rc = b->dalloc(&b->y, sizeof(float) * R * b->ldy)) ||
        (rc = b->dalloc(&b->qbuf, sizeof(float) * R * c->nq * c->hd)) ||
        (rc = b->dalloc(&b->act_h.q, R * c->H)) || (rc = b->dalloc(&b->act_h.d, sizeof(float) * R * (c->H / 32))) ||
        (rc = b->dalloc(&b->act_h.fs, sizeof(float) * R * (c->H / 32))) ||
        (rc = b->dalloc(&b->act_mid.q, R * mid)) || (rc = b->dalloc(&b->act_mid.d, sizeof(float) * R * (mid / 32))) ||
        (rc = b->dalloc(&b->act_mid.fs, sizeof(float) * R * (mid / 32))) ||
        (rc = b->dalloc(&b->partial, sizeof(unsigned long long) * R * b->head.npanels)) ||
        (rc = b->dalloc(&b->nan0, sizeof(int) * R)) || (rc = b->dalloc(&b->status, sizeof(int))) ||
        (rc = b->dalloc(&b->dn_recs, sizeof(float) * deltanet_rec_floats(b->lind, (int)R))) ||
        (rc = b->dalloc(&b->dn_o, sizeof(float) * R * c->vd)) ||
        (rc = b->dalloc(&b->keys, sizeof(unsigned long long) * 2 * R)) ||
        (rc = b->dalloc(&b->steps, sizeof(Step) * S)) || (rc = b->dalloc(&b->d_seeds, sizeof(unsigned long long) * S)) ||
        (rc = b->dalloc(&b->d_ndone, sizeof(int))))
        return rc;
    b->act_h.cols = c->H;
    // defined contents for rows a pass does not write (padding rows of finished sequences)
    NB_CUDA_OK(cudaMemsetAsync(b->x, 0, sizeof(float) * R * c->H, b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->y, 0, sizeof(float) * R * b->ldy, b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->act_h.q, 0, R * c->H, b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->act_h.d, 0, sizeof(float) * R * (c->H / 32), b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->act_h.fs, 0, sizeof(float) * R * (c->H / 32), b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->act_mid.q, 0, R * mid, b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->act_mid.d, 0, sizeof(float) * R * (mid / 32), b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->act_mid.fs, 0, sizeof(float) * R * (mid / 32), b->stream));
    NB_CUDA_OK(cudaMemsetAsync(b->nan0, 0, sizeof(int) * R, b->stream));   // only vocabulary row 0's shard sets it
    if (gemm_maps(b->act_h, (int)R, &b->maps_h) || gemm_maps(with_cols(b->act_mid, c->vd), (int)R, &b->maps_ol) ||
        gemm_maps(with_cols(b->act_mid, c->nq * c->hd), (int)R, &b->maps_oa) ||
        gemm_maps(with_cols(b->act_mid, c->ffn), (int)R, &b->maps_f))
        return PINFER_E_NOMEM;
    // host-chosen pass shapes: one slot of S per prefill step (the host fills slot i while the
    // device may still read slot i - 1)
    b->pass_slots = (b->max_ctx + kMaxRows - 1) / kMaxRows + 2;
    if ((rc = b->dalloc(&b->d_pass, sizeof(SeqPass) * S * b->pass_slots))) return rc;
    NB_CUDA_OK(cudaMallocHost(&b->h_pass, sizeof(SeqPass) * S * b->pass_slots));
    NB_CUDA_OK(cudaMallocHost(&b->h_steps, sizeof(Step) * S));
    NB_CUDA_OK(cudaMallocHost(&b->h_ndone, sizeof(int)));
    NB_CUDA_OK(cudaMemsetAsync(b->status, 0, sizeof(int), b->stream));
    NB_CUDA_OK(cudaStreamSynchronize(b->stream));
    return PINFER_OK;
}

int ensure_out(pinfer_b200_batch *b, size_t n) {
    if (b->out_cap >= n) return PINFER_OK;
    int rc;
    if ((rc = b->dalloc(&b->d_out, sizeof(int) * n)) || (rc = b->dalloc(&b->d_greedy, sizeof(int) * n))) return rc;
    b->out_cap = n;
    return PINFER_OK;
}

// The verify round of nseq sequences at draft depth k: one pass of k + 1 rows per sequence,
// greedy acceptance and commit, the count of finished sequences.
int round_graph(pinfer_b200_batch *b, int nseq, int k, cudaGraphExec_t *out) {
    if (b->graph && (b->graph_nseq != nseq || b->graph_k != k || b->graph_out != b->d_out)) {
        cudaGraphExecDestroy(b->graph);
        b->graph = nullptr;
    }
    if (!b->graph) {
        cudaGraph_t g;
        NB_CUDA_OK(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
        enqueue_forward(b, nseq * (k + 1), nseq, k + 1, true);
        launch_accept(b->steps, b->d_greedy, b->d_out, b->stream, nseq);
        launch_count_done(b->steps, nseq, b->d_ndone, b->stream);
        NB_CUDA_OK(cudaStreamEndCapture(b->stream, &g));
        const cudaError_t e = cudaGraphInstantiate(&b->graph, g, 0);
        cudaGraphDestroy(g);
        NB_CUDA_OK(e);
        b->graph_nseq = nseq;
        b->graph_k = k;
        b->graph_out = b->d_out;
    }
    *out = b->graph;
    return PINFER_OK;
}

}  // namespace

extern "C" {

pinfer_b200_batch *pinfer_b200_batch_create(pinfer_ctx *ctx, int slots, int max_ctx, int max_k, int *err) {
    int dummy;
    if (!err) err = &dummy;
    *err = PINFER_E_ARG;
    if (!ctx || slots < 1 || slots > 2048 || max_k < 0 || max_k >= kMaxRows || max_ctx < 2 ||
        max_ctx > ctx->max_ctx)
        return nullptr;
    if (cudaSetDevice(ctx->device) != cudaSuccess) {
        *err = PINFER_E_NOMEM;
        return nullptr;
    }
    pinfer_b200_batch *b = new (std::nothrow) pinfer_b200_batch();
    if (!b) {
        *err = PINFER_E_NOMEM;
        return nullptr;
    }
    b->src = ctx;
    b->weights = ctx->weights;
    b->device = ctx->device;
    b->S = slots;
    b->max_ctx = max_ctx;
    b->kmax = max_k;
    const int rc = batch_alloc(b);
    if (rc) {
        delete b;
        *err = rc;
        return nullptr;
    }
    *err = PINFER_OK;
    return b;
}

void *pinfer_b200_batch_stream(pinfer_b200_batch *b) { return b ? (void *)b->stream : nullptr; }

int pinfer_b200_batch_rounds(const pinfer_b200_batch *b) { return b ? b->last_rounds : -1; }

void pinfer_b200_batch_free(pinfer_b200_batch *b) {
    if (!b) return;
    cudaSetDevice(b->device);
    cudaStreamSynchronize(b->stream);
    delete b;
}

int pinfer_b200_batch_generate_synthetic(pinfer_b200_batch *b, int n_seq, const int32_t *prompts,
                                         const int32_t *prompt_lens, int n_max, int k, const int32_t *greedy,
                                         const uint64_t *seeds, float p, int32_t *out, int32_t *counts,
                                         int32_t *status, pinfer_spec_stats *stats, float *decode_ms) {
    if (!b || n_seq < 1 || n_seq > b->S || !prompts || !prompt_lens || n_max < 1 || k < 0 || k > b->kmax ||
        (k > 0 && (!greedy || !seeds)) || !(p >= 0.0f && p <= 1.0f) || !out || !counts)
        return PINFER_E_ARG;
    const pinfer_ctx *c = b->src;
    std::vector<size_t> off(n_seq + 1, 0);
    for (int i = 0; i < n_seq; i++) {
        if (prompt_lens[i] < 1) return PINFER_E_ARG;
        if (prompt_lens[i] >= b->max_ctx) return PINFER_E_CTX_FULL;
        off[i + 1] = off[i] + (size_t)prompt_lens[i];
    }
    for (size_t i = 0; i < off[n_seq]; i++)
        if (prompts[i] < 0 || prompts[i] >= c->vocab) return PINFER_E_ARG;
    NB_CUDA_OK(cudaSetDevice(b->device));
    cudaStream_t s = b->stream;
    int rc;
    if ((rc = ensure_out(b, (size_t)n_seq * n_max))) return rc;
    if (k > 0) {
        NB_CUDA_OK(cudaMemcpyAsync(b->d_greedy, greedy, sizeof(int) * (size_t)n_seq * n_max, cudaMemcpyHostToDevice, s));
        NB_CUDA_OK(cudaMemcpyAsync(b->d_seeds, seeds, sizeof(unsigned long long) * n_seq, cudaMemcpyHostToDevice, s));
    }
    // fresh states (the KV rows are written before they are read)
    for (int l = 0; l < c->n_layers; l++) {
        if (c->layers[l].is_full) continue;
        const LinLayer &N = b->lin[c->layers[l].lin];
        NB_CUDA_OK(cudaMemsetAsync(N.conv_state, 0, sizeof(float) * n_seq * b->lind.ss_conv, s));
        NB_CUDA_OK(cudaMemsetAsync(N.rec, 0, sizeof(float) * n_seq * b->lind.ss_rec, s));
    }
    NB_CUDA_OK(cudaMemsetAsync(b->steps, 0, sizeof(Step) * n_seq, s));
    NB_CUDA_OK(cudaMemsetAsync(b->status, 0, sizeof(int), s));
    GenArgs g{};
    g.n_max = n_max;
    g.k = k;
    g.eos = c->eos;
    g.n_stop = 0;
    g.max_ctx = b->max_ctx;
    g.vocab = c->vocab;
    g.drafter = 0;
    g.p24 = (unsigned)std::min(16777216.0, std::floor((double)p * 16777216.0 + 0.5));
    g.seed = 0;
    launch_set_gen(b->steps, g, s, n_seq, k > 0 ? b->d_seeds : nullptr);

    // prefill: every prompt but its last token, up to kMaxRows rows per sequence per pass
    std::vector<int> fed(n_seq, 0);
    int slot = 0;
    auto set_passes = [&](int R_unused) -> int {
        (void)R_unused;
        SeqPass *hp = b->h_pass + (size_t)slot * b->S;
        SeqPass *dp = b->d_pass + (size_t)slot * b->S;
        NB_CUDA_OK(cudaMemcpyAsync(dp, hp, sizeof(SeqPass) * n_seq, cudaMemcpyHostToDevice, s));
        launch_set_pass_seqs(b->steps, dp, n_seq, s);
        slot = (slot + 1) % b->pass_slots;
        return PINFER_OK;
    };
    for (;;) {
        if (slot == 0) NB_CUDA_OK(cudaStreamSynchronize(s));   // the ring wrapped: its slots are free again
        SeqPass *hp = b->h_pass + (size_t)slot * b->S;
        int R = 0, rps = 0;
        for (int i = 0; i < n_seq; i++) {
            const int left = prompt_lens[i] - 1 - fed[i];
            const int n = std::min(kMaxRows, std::max(left, 0));
            hp[i].n = n;
            hp[i].pos0 = fed[i];
            hp[i].row0 = R;
            hp[i].logged = 0;
            for (int t = 0; t < n; t++) hp[i].tokens[t] = prompts[off[i] + fed[i] + t];
            fed[i] += n;
            R += n;
            rps = std::max(rps, n);
        }
        if (R == 0) break;
        if ((rc = set_passes(R))) return rc;
        enqueue_forward(b, R, n_seq, rps, false, true);
    }
    // the last prompt token of every sequence, with the LM head: the first generated token
    {
        if (slot == 0) NB_CUDA_OK(cudaStreamSynchronize(s));
        SeqPass *hp = b->h_pass + (size_t)slot * b->S;
        for (int i = 0; i < n_seq; i++) {
            hp[i].n = 1;
            hp[i].pos0 = prompt_lens[i] - 1;
            hp[i].row0 = i * (k + 1);
            hp[i].logged = 0;
            hp[i].tokens[0] = prompts[off[i + 1] - 1];
        }
        if ((rc = set_passes(n_seq))) return rc;
        enqueue_forward(b, n_seq * (k + 1), n_seq, 1, true);
        launch_gen_start(b->steps, k > 0 ? b->d_greedy : nullptr, b->d_out, s, n_seq);
    }
    NB_CUDA_OK(cudaGetLastError());
    // verify rounds (row0 = i (k + 1) stays from the pass above)
    cudaGraphExec_t ex;
    if ((rc = round_graph(b, n_seq, k, &ex))) return rc;
    cudaEvent_t ev0, ev1;
    NB_CUDA_OK(cudaEventCreate(&ev0));
    NB_CUDA_OK(cudaEventCreate(&ev1));
    cudaEventRecord(ev0, s);
    int rounds = 0;
    const int max_rounds = n_max + 2;   // every round emits a token of each live sequence
    for (;;) {
        const int reps = std::min(std::max(1, (n_max - rounds) / (k + 1) / 2), 16);
        for (int i = 0; i < reps && rounds < max_rounds; i++, rounds++) {
            if (cudaGraphLaunch(ex, s) != cudaSuccess) {
                cudaEventDestroy(ev0);
                cudaEventDestroy(ev1);
                set_last_error("pinfer_b200_batch: graph launch failed");
                return PINFER_E_NOMEM;
            }
        }
        cudaMemcpyAsync(b->h_ndone, b->d_ndone, sizeof(int), cudaMemcpyDeviceToHost, s);
        if (cudaStreamSynchronize(s) != cudaSuccess) {
            cudaEventDestroy(ev0);
            cudaEventDestroy(ev1);
            set_last_error("pinfer_b200_batch: a round failed on the device");
            return PINFER_E_NOMEM;
        }
        if (*b->h_ndone >= n_seq || rounds >= max_rounds) break;
    }
    cudaEventRecord(ev1, s);
    cudaEventSynchronize(ev1);
    b->last_rounds = rounds;
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    cudaEventDestroy(ev0);
    cudaEventDestroy(ev1);
    if (decode_ms) *decode_ms = ms;
    int dstat = 0;
    NB_CUDA_OK(cudaMemcpy(&dstat, b->status, sizeof(int), cudaMemcpyDeviceToHost));
    NB_CUDA_OK(cudaMemcpy(b->h_steps, b->steps, sizeof(Step) * n_seq, cudaMemcpyDeviceToHost));
    NB_CUDA_OK(cudaMemcpy(out, b->d_out, sizeof(int) * (size_t)n_seq * n_max, cudaMemcpyDeviceToHost));
    for (int i = 0; i < n_seq; i++) {
        const Step &st = b->h_steps[i];
        counts[i] = st.count;
        if (status) status[i] = st.done ? st.status : PINFER_E_NOMEM;
        if (stats) {
            stats->rounds += st.rounds;
            stats->drafted += st.drafted;
            stats->accepted += st.accepted;
        }
    }
    if (dstat) {
        set_last_error("pinfer_b200_batch: a bounded device wait timed out in the tensor-core GEMM");
        return PINFER_E_NOMEM;
    }
    return PINFER_OK;
}

}  // extern "C"
