// Prefill of a single context through the tensor-core GEMMs: the prompt's rows in chunks of up
// to kPrefillRows (64), as the reference's batched prefill (pf_forward_h, engine/src/forward.c:
// 154-165: chunks of ctx->batch <= 64 rows, each projection one pf_matmul that reads the weights
// once for the whole chunk, engine/src/matvec_fast.c:469-550).
//
// A chunk of R rows is one pass: the embedding and every RMSNorm + A8 over the R rows, each
// projection one tcgen05 GEMM over them (the weights' tile image read once per chunk), the
// SwiGLU + A8 between gate / up and down. A Gated DeltaNet layer runs the chunk's rows in order
// (k_deltanet_prep / _rows / _post: the conv, norms and gates of all rows in parallel,
// the sequential recurrence with its state in registers, the gated norms in parallel).
// An attention layer sees the chunk as consecutive 16-row sub-passes, Step blocks with
// row0 = 16 i and pos0 = n_past + 16 i over the context's one KV cache (no per-sequence
// stride): k_attn_prep writes the K / V rows of the whole chunk, then every row attends to the
// positions up to its own (k_attn5 with one row per CTA: the group's query heads share each
// K / V row). Every row's arithmetic is the 16-row CUDA-core path's, so logits, states and
// later tokens are bit-identical to it, and to the reference.
#include <algorithm>
#include <vector>

#include "nb_ctx.h"

using namespace nb;

namespace {

int tile_into(pinfer_ctx *c, const Mat &W0, const Mat &W1, GemmW *out) {
    const int rows = W1.npanels ? W0.npanels * kPanelRows + W1.rows : W0.rows;
    uint8_t *t = nullptr;
    int rc = c->dalloc(&t, gemm_tiled_bytes(rows, W0.cols), true);
    if (rc) return rc;
    launch_gemm_tile(W0, W1, t, c->stream);
    *out = gemm_w(W0, W1, t);
    return PINFER_OK;
}

Act with_cols(Act a, int cols) {
    a.cols = cols;
    return a;
}

int prefill_alloc(pinfer_ctx *c, bool logits) {
    PrefillScratch &p = c->pf;
    const size_t R = kPrefillRows;
    int rc;
    if (!p.ready) {
        p.ldy = std::max(std::max(c->lind.ldy, c->attd.ldy), 2 * c->ffn);
        const int mid = std::max(std::max(c->vd, c->nq * c->hd), c->ffn);
        const size_t chunks = ((size_t)c->max_ctx + kPrefillRows - 1) / kPrefillRows;
        if ((rc = c->dalloc(&p.x, sizeof(float) * R * c->H)) || (rc = c->dalloc(&p.y, sizeof(float) * R * p.ldy)) ||
            (rc = c->dalloc(&p.qbuf, sizeof(float) * R * c->nq * c->hd)) || (rc = c->dalloc(&p.act_h.q, R * c->H)) ||
            (rc = c->dalloc(&p.act_h.d, sizeof(float) * R * (c->H / 32))) ||
            (rc = c->dalloc(&p.act_h.fs, sizeof(float) * R * (c->H / 32))) ||
            (rc = c->dalloc(&p.act_mid.q, R * mid)) || (rc = c->dalloc(&p.act_mid.d, sizeof(float) * R * (mid / 32))) ||
            (rc = c->dalloc(&p.act_mid.fs, sizeof(float) * R * (mid / 32))) ||
            (rc = c->dalloc(&p.steps, sizeof(Step) * kPrefillSub)) ||
            (rc = c->dalloc(&p.dn_recs, sizeof(float) * deltanet_rec_floats(c->lind, (int)R))) ||
            (rc = c->dalloc(&p.dn_o, sizeof(float) * R * c->vd)) ||
            (rc = c->dalloc(&p.d_pass, sizeof(SeqPass) * kPrefillSub * chunks)))
            return rc;
        p.act_h.cols = c->H;
        if (gemm_maps(p.act_h, (int)R, &p.maps_h) || gemm_maps(with_cols(p.act_mid, c->vd), (int)R, &p.maps_ol) ||
            gemm_maps(with_cols(p.act_mid, c->nq * c->hd), (int)R, &p.maps_oa) ||
            gemm_maps(with_cols(p.act_mid, c->ffn), (int)R, &p.maps_f))
            return PINFER_E_NOMEM;
        p.ready = true;
    }
    if (logits && !p.logits) {
        const int npanels = (c->vocab + kPanelRows - 1) / kPanelRows;
        if ((rc = c->dalloc(&p.logits, sizeof(float) * R * (size_t)c->vocab)) ||
            (rc = c->dalloc(&p.partial, sizeof(unsigned long long) * R * npanels)) ||
            (rc = c->dalloc(&p.nan0, sizeof(int) * R)))
            return rc;
    }
    return PINFER_OK;
}

void pf_gemm(pinfer_ctx *c, int epi, const GemmMaps &maps, const GemmW &W, int R, float *y, int ldy) {
    GemmArgs g;
    g.W = W;
    g.n = R;
    g.y = y;
    g.ldy = ldy;
    g.partial = c->pf.partial;
    g.nan0 = c->pf.nan0;
    g.row_base = 0;
    g.status = &c->step->status;   // a bounded wait that gave up is reported like the passes'
    launch_gemm(epi, maps, g, c->stream);
}

// One chunk of R rows whose sub-pass shapes are in p.steps (set by the caller).
void enqueue_chunk(pinfer_ctx *c, int R, bool logits) {
    PrefillScratch &p = c->pf;
    const WeightStore &ws = *c->weights;
    cudaStream_t s = c->stream;
    const int nsub = (R + kMaxRows - 1) / kMaxRows;
    AttnDims ad = c->attd;
    ad.rps = kMaxRows;
    ad.ss_kv = 0;   // every sub-pass reads and writes the one cache
    launch_embed(c->embed, p.steps, p.x, c->H, s, nsub, kMaxRows);
    for (int l = 0; l < c->n_layers; l++) {
        const auto &D = c->layers[l];
        const auto &T = ws.tiles[l];
        launch_norm_quant(p.x, D.in_norm, c->H, c->eps, p.steps, p.act_h, s, nsub, kMaxRows);
        if (D.is_full) {
            pf_gemm(c, 0, p.maps_h, T.win, R, p.y, c->attd.ldy);
            const Act o = with_cols(p.act_mid, c->nq * c->hd);
            launch_attn_prep(c->att[l], ad, p.y, p.qbuf, p.steps, s, nsub);
            launch_attn_rows(c->att[l], ad, p.y, p.qbuf, p.steps, o, s, nsub);
            pf_gemm(c, 1, p.maps_oa, T.out, R, p.x, c->H);
        } else {
            pf_gemm(c, 0, p.maps_h, T.win, R, p.y, c->lind.ldy);
            const Act o = with_cols(p.act_mid, c->vd);
            launch_deltanet_rows(c->lin[D.lin], c->lind, p.y, R, p.dn_recs, p.dn_o, o, &c->step->status, s);
            pf_gemm(c, 1, p.maps_ol, T.out, R, p.x, c->H);
        }
        launch_norm_quant(p.x, D.post_norm, c->H, c->eps, p.steps, p.act_h, s, nsub, kMaxRows);
        pf_gemm(c, 0, p.maps_h, T.gu, R, p.y, 2 * c->ffn);
        launch_swiglu_quant(p.y, 2 * c->ffn, c->ffn, R, with_cols(p.act_mid, c->ffn), s);
        pf_gemm(c, 1, p.maps_f, T.down, R, p.x, c->H);
    }
    if (logits) {
        launch_norm_quant(p.x, c->norm, c->H, c->eps, p.steps, p.act_h, s, nsub, kMaxRows);
        pf_gemm(c, 4, p.maps_h, ws.head_tile, R, p.logits, c->vocab);
    }
}

}  // namespace

int ensure_gemm_tiles(pinfer_ctx *c, bool head) {
    WeightStore &ws = *c->weights;
    std::lock_guard<std::mutex> lock(ws.tile_mu);
    int rc;
    if (!ws.tiles_ok) {
        const Mat none;
        for (int l = 0; l < c->n_layers; l++) {
            const auto &D = c->layers[l];
            auto &T = ws.tiles[l];
            if ((rc = tile_into(c, D.win, none, &T.win)) || (rc = tile_into(c, D.out, none, &T.out)) ||
                (rc = tile_into(c, D.gate, D.up, &T.gu)) || (rc = tile_into(c, D.down, none, &T.down)))
                return rc;
        }
        NB_CUDA_OK(cudaStreamSynchronize(c->stream));   // other contexts' streams use them next
        ws.tiles_ok = true;
    }
    if (head && !ws.head_tile_ok) {
        if ((rc = tile_into(c, c->head, Mat(), &ws.head_tile))) return rc;
        NB_CUDA_OK(cudaStreamSynchronize(c->stream));
        ws.head_tile_ok = true;
    }
    return PINFER_OK;
}

bool prefill_gemm_ok(const pinfer_ctx *c) {
    return deltanet_batch_ok(c->lind) && attn_batch_ok(c->attd);
}

int prefill_gemm(pinfer_ctx *c, const int32_t *tokens, int n, float *logits_all) {
    const bool logits = logits_all != nullptr;
    int rc;
    if (logits && c->shard_world > 1) return PINFER_E_ARG;   // the sharded head has no whole tile
    if ((rc = ensure_gemm_tiles(c, logits)) || (rc = prefill_alloc(c, logits))) return rc;
    PrefillScratch &p = c->pf;
    cudaStream_t s = c->stream;
    // a deferred commit of the last generation is applied first: k_deltanet_rows replays none
    launch_flush(c->lin, c->n_lin, c->lind, c->step, s);
    // every chunk's sub-pass shapes in one copy (a pageable source: staged before the call returns)
    const int nchunks = (n + kPrefillRows - 1) / kPrefillRows;
    std::vector<SeqPass> hp((size_t)nchunks * kPrefillSub);
    for (int j = 0; j < nchunks; j++)
        for (int i = 0; i < kPrefillSub; i++) {
            const int t0 = j * kPrefillRows + i * kMaxRows;
            SeqPass &q = hp[(size_t)j * kPrefillSub + i];
            q.n = std::max(0, std::min(kMaxRows, n - t0));
            q.pos0 = c->n_past + t0;
            q.row0 = i * kMaxRows;
            q.logged = 0;
            for (int t = 0; t < q.n; t++) q.tokens[t] = tokens[t0 + t];
        }
    NB_CUDA_OK(cudaMemcpyAsync(p.d_pass, hp.data(), sizeof(SeqPass) * hp.size(), cudaMemcpyHostToDevice, s));
    for (int j = 0; j < nchunks; j++) {
        const int R = std::min(kPrefillRows, n - j * kPrefillRows);
        launch_set_pass_seqs(p.steps, p.d_pass + (size_t)j * kPrefillSub, (R + kMaxRows - 1) / kMaxRows, s);
        enqueue_chunk(c, R, logits);
        if (logits)
            NB_CUDA_OK(cudaMemcpyAsync(logits_all + (size_t)j * kPrefillRows * c->vocab, p.logits,
                                       sizeof(float) * (size_t)R * c->vocab, cudaMemcpyDeviceToHost, s));
    }
    c->n_past += n;
    NB_CUDA_OK(cudaGetLastError());
    return PINFER_OK;
}
