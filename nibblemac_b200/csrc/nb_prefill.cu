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
            (rc = c->dalloc(&p.d_pass, sizeof(SeqPass) * kPrefillSub * chunks * 2)))
            return rc;
        p.act_h.cols = c->H;
        if (c->mtp_ok) {
            if ((rc = c->dalloc(&p.hn, sizeof(float) * R * c->H)) ||
                (rc = c->dalloc(&p.msteps, sizeof(Step) * kPrefillSub)) ||
                (rc = c->dalloc(&p.act_cat.q, R * 2 * c->H)) ||
                (rc = c->dalloc(&p.act_cat.d, sizeof(float) * R * (2 * c->H / 32))) ||
                (rc = c->dalloc(&p.act_cat.fs, sizeof(float) * R * (2 * c->H / 32))))
                return rc;
            p.act_cat.cols = 2 * c->H;
            if (gemm_maps(p.act_cat, (int)R, &p.maps_cat)) return PINFER_E_NOMEM;
        }
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

// A full-attention decoder block over the chunk's R rows (sub-passes st), its KV cache in A.
void attention_block(pinfer_ctx *c, const pinfer_ctx::Layer &D, const WeightStore::TileLayer &T,
                     const AttnLayer &A, const Step *st, int R) {
    PrefillScratch &p = c->pf;
    cudaStream_t s = c->stream;
    const int nsub = (R + kMaxRows - 1) / kMaxRows;
    AttnDims ad = c->attd;
    ad.rps = kMaxRows;
    ad.ss_kv = 0;   // every sub-pass reads and writes the one cache
    launch_norm_quant(p.x, D.in_norm, c->H, c->eps, st, p.act_h, s, nsub, kMaxRows);
    pf_gemm(c, 0, p.maps_h, T.win, R, p.y, c->attd.ldy);
    const Act o = with_cols(p.act_mid, c->nq * c->hd);
    launch_attn_prep(A, ad, p.y, p.qbuf, st, s, nsub);
    launch_attn_rows(A, ad, p.y, p.qbuf, st, o, s, nsub);
    pf_gemm(c, 1, p.maps_oa, T.out, R, p.x, c->H);
    launch_norm_quant(p.x, D.post_norm, c->H, c->eps, st, p.act_h, s, nsub, kMaxRows);
    pf_gemm(c, 0, p.maps_h, T.gu, R, p.y, 2 * c->ffn);
    launch_swiglu_quant(p.y, 2 * c->ffn, c->ffn, R, with_cols(p.act_mid, c->ffn), s);
    pf_gemm(c, 1, p.maps_f, T.down, R, p.x, c->H);
}

// One chunk of R rows whose sub-pass shapes are in p.steps (set by the caller); with mtp, the
// MTP head's pass over the same rows follows (its sub-passes in p.msteps: the next tokens):
// u = fc [rmsnorm(embed(next)) | rmsnorm(final-normed row)], then its decoder block, which
// writes the MTP KV rows (pf_spec_prefill, spec.c:172-195; pf_mtp_forward, mtp.c:62-100).
void enqueue_chunk(pinfer_ctx *c, int R, bool logits, bool mtp) {
    PrefillScratch &p = c->pf;
    const WeightStore &ws = *c->weights;
    cudaStream_t s = c->stream;
    const int nsub = (R + kMaxRows - 1) / kMaxRows;
    launch_embed(c->embed, p.steps, p.x, c->H, s, nsub, kMaxRows);
    for (int l = 0; l < c->n_layers; l++) {
        const auto &D = c->layers[l];
        const auto &T = ws.tiles[l];
        if (D.is_full) {
            attention_block(c, D, T, c->att[l], p.steps, R);
            continue;
        }
        launch_norm_quant(p.x, D.in_norm, c->H, c->eps, p.steps, p.act_h, s, nsub, kMaxRows);
        pf_gemm(c, 0, p.maps_h, T.win, R, p.y, c->lind.ldy);
        const Act o = with_cols(p.act_mid, c->vd);
        launch_deltanet_rows(c->lin[D.lin], c->lind, p.y, R, p.dn_recs, p.dn_o, o, &c->step->status, s);
        pf_gemm(c, 1, p.maps_ol, T.out, R, p.x, c->H);
        launch_norm_quant(p.x, D.post_norm, c->H, c->eps, p.steps, p.act_h, s, nsub, kMaxRows);
        pf_gemm(c, 0, p.maps_h, T.gu, R, p.y, 2 * c->ffn);
        launch_swiglu_quant(p.y, 2 * c->ffn, c->ffn, R, with_cols(p.act_mid, c->ffn), s);
        pf_gemm(c, 1, p.maps_f, T.down, R, p.x, c->H);
    }
    if (mtp) {
        launch_norm_rows(p.x, c->norm, c->H, c->eps, p.steps, p.hn, s, nsub);
        launch_mtp_input(c->embed, p.hn, p.msteps, c->mtp_norm_emb, c->mtp_norm_hid, c->H, c->eps, p.act_cat, s,
                         nsub);
        pf_gemm(c, 0, p.maps_cat, ws.mtp_fc_tile, R, p.x, c->H);
        attention_block(c, c->mtp_layer, ws.mtp_tiles, c->mtp_att, p.msteps, R);
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
        if (c->mtp_ok) {
            const auto &D = c->mtp_layer;
            auto &T = ws.mtp_tiles;
            if ((rc = tile_into(c, D.win, none, &T.win)) || (rc = tile_into(c, D.out, none, &T.out)) ||
                (rc = tile_into(c, D.gate, D.up, &T.gu)) || (rc = tile_into(c, D.down, none, &T.down)) ||
                (rc = tile_into(c, c->mtp_fc, none, &ws.mtp_fc_tile)))
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

int prefill_gemm(pinfer_ctx *c, const int32_t *tokens, int n, float *logits_all, const int32_t *next) {
    const bool logits = logits_all != nullptr, mtp = next != nullptr;
    int rc;
    if (logits && c->shard_world > 1) return PINFER_E_ARG;   // the sharded head has no whole tile
    if ((mtp && !c->mtp_ok) || (mtp && logits)) return PINFER_E_ARG;   // the MTP pass reuses the rows
    if ((rc = ensure_gemm_tiles(c, logits)) || (rc = prefill_alloc(c, logits))) return rc;
    PrefillScratch &p = c->pf;
    cudaStream_t s = c->stream;
    // a deferred commit of the last generation is applied first: k_deltanet_rows replays none
    launch_flush(c->lin, c->n_lin, c->lind, c->step, s);
    // every chunk's sub-pass shapes in one copy (a pageable source: staged before the call returns)
    // (the MTP sub-passes, with the next tokens, after the main ones)
    const int nchunks = (n + kPrefillRows - 1) / kPrefillRows;
    const size_t nmain = (size_t)nchunks * kPrefillSub;
    std::vector<SeqPass> hp(nmain * (mtp ? 2 : 1));
    for (int j = 0; j < nchunks; j++)
        for (int i = 0; i < kPrefillSub; i++) {
            const int t0 = j * kPrefillRows + i * kMaxRows;
            SeqPass &q = hp[(size_t)j * kPrefillSub + i];
            q.n = std::max(0, std::min(kMaxRows, n - t0));
            q.pos0 = c->n_past + t0;
            q.row0 = i * kMaxRows;
            q.logged = 0;
            for (int t = 0; t < q.n; t++) q.tokens[t] = tokens[t0 + t];
            if (mtp) {
                SeqPass &m = hp[nmain + (size_t)j * kPrefillSub + i];
                m = q;
                for (int t = 0; t < q.n; t++) m.tokens[t] = next[t0 + t];
            }
        }
    NB_CUDA_OK(cudaMemcpyAsync(p.d_pass, hp.data(), sizeof(SeqPass) * hp.size(), cudaMemcpyHostToDevice, s));
    for (int j = 0; j < nchunks; j++) {
        const int R = std::min(kPrefillRows, n - j * kPrefillRows);
        const int nsub = (R + kMaxRows - 1) / kMaxRows;
        launch_set_pass_seqs(p.steps, p.d_pass + (size_t)j * kPrefillSub, nsub, s);
        if (mtp) launch_set_pass_seqs(p.msteps, p.d_pass + nmain + (size_t)j * kPrefillSub, nsub, s);
        enqueue_chunk(c, R, logits, mtp);
        if (logits)
            NB_CUDA_OK(cudaMemcpyAsync(logits_all + (size_t)j * kPrefillRows * c->vocab, p.logits,
                                       sizeof(float) * (size_t)R * c->vocab, cudaMemcpyDeviceToHost, s));
    }
    c->n_past += n;
    NB_CUDA_OK(cudaGetLastError());
    return PINFER_OK;
}
