// pinfer C API on the B200 (host side): model upload, forward-pass orchestration, the
// speculative verify / accept loop as a replayed CUDA graph, and the reference's API surface
// (engine/include/pinfer.h). The device does every model computation; the host validates
// arguments exactly as the reference does, launches work and copies results out.
#include <sys/sysinfo.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>
#include <new>

#include "nb_engine.h"
#include "nb_model.h"
#include "nb_nccl.h"
#include "pinfer.h"
#include "nb_b200.h"

using namespace nb;

namespace {

thread_local std::string g_err;

void set_err(const char *msg) {
    g_err = msg;
    fprintf(stderr, "pinfer: %s\n", msg);
}

#define CUDA_OK(call)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            char b_[256];                                                              \
            snprintf(b_, sizeof b_, "CUDA error %s at %s:%d", cudaGetErrorString(e_),  \
                     __FILE__, __LINE__);                                              \
            set_err(b_);                                                               \
            return PINFER_E_NOMEM;                                                     \
        }                                                                              \
    } while (0)

}  // namespace

// ---------------------------------------------------------------- panel repack
namespace nb {

void set_last_error(const char *msg) { set_err(msg); }

size_t panel_bytes(int rows, int cols) {
    const size_t np = ((size_t)rows + kPanelRows - 1) / kPanelRows;
    return np * (size_t)(cols / 256) * kUnitBytes;
}

// Write rows [0, rows) of a .pq Q4K matrix into a panel buffer at row offset `row0`
// (a multiple of 4). Codes and scale values are moved, never changed.
static void repack_into(const uint8_t *pq, int rows, int cols, uint8_t *out, int row0) {
    const int nsb = cols / 256;
    for (int r = 0; r < rows; r++) {
        const int dr = row0 + r, panel = dr / kPanelRows, lane = dr % kPanelRows;
        const uint8_t *tile = pq + (size_t)(r / 4) * nsb * 576;
        const int i = r % 4;
        for (int sb = 0; sb < nsb; sb++) {
            const uint8_t *p = tile + (size_t)sb * 576;
            uint8_t *u = out + ((size_t)panel * nsb + sb) * kUnitBytes;
            uint16_t D, M;
            memcpy(&D, p + 2 * i, 2);
            memcpy(&M, p + 8 + 2 * i, 2);
            uint64_t A = (uint64_t)D << 48, B = (uint64_t)M << 48;
            for (int k = 0; k < 8; k++) {
                const int j = 4 * k + i;   // 6-bit arrays are [block][row]
                auto get6 = [&](const uint8_t *q) {
                    const int lo = j < 16 ? q[j] & 15 : q[j - 16] >> 4;
                    return (uint64_t)(lo | ((q[16 + j % 8] >> (2 * (j / 8))) & 3) << 4);
                };
                A |= get6(p + 16) << (6 * k);
                B |= get6(p + 40) << (6 * k);
            }
            memcpy(u + 16 * lane, &A, 8);
            memcpy(u + 16 * lane + 8, &B, 8);
            for (int k = 0; k < 8; k++)
                memcpy(u + 512 * (k + 1) + 16 * lane, p + 64 + 64 * k + 16 * i, 16);
        }
    }
}

void repack_q4k(const uint8_t *pq, int rows, int cols, uint8_t *out) {
    memset(out, 0, panel_bytes(rows, cols));
    repack_into(pq, rows, cols, out, 0);
}

}  // namespace nb

#include "nb_ctx.h"

namespace {

int upload_floats(pinfer_ctx *c, const float *h, size_t n, float **d) {
    int rc = c->dalloc(d, n * sizeof(float), true);
    if (rc) return rc;
    CUDA_OK(cudaMemcpy(*d, h, n * sizeof(float), cudaMemcpyHostToDevice));
    return PINFER_OK;
}

// Concatenate Q4K matrices (same column count) by rows into one panel-layout matrix.
int upload_mats(pinfer_ctx *c, const PqMat *const *parts, int nparts, Mat *out) {
    int rows = 0;
    const int cols = parts[0]->cols;
    for (int i = 0; i < nparts; i++) rows += parts[i]->rows;
    const size_t bytes = panel_bytes(rows, cols);
    std::vector<uint8_t> buf(bytes, 0);
    int r0 = 0;
    for (int i = 0; i < nparts; i++) {
        repack_into(parts[i]->data, parts[i]->rows, cols, buf.data(), r0);
        r0 += parts[i]->rows;
    }
    uint8_t *d = nullptr;
    int rc = c->dalloc(&d, bytes, true);
    if (rc) return rc;
    CUDA_OK(cudaMemcpy(d, buf.data(), bytes, cudaMemcpyHostToDevice));
    out->w = d;
    out->rows = rows;
    out->cols = cols;
    out->npanels = (rows + kPanelRows - 1) / kPanelRows;
    out->nsb = cols / 256;
    return PINFER_OK;
}

int upload_mat(pinfer_ctx *c, const PqMat &m, Mat *out) {
    const PqMat *p = &m;
    return upload_mats(c, &p, 1, out);
}

void set_dims(pinfer_ctx *c) {
    const PqHeader *h = c->file.hdr;
    c->H = (int)h->hidden;
    c->ffn = (int)h->ffn;
    c->n_layers = (int)h->n_layers;
    c->vocab = (int)h->vocab;
    c->nq = (int)h->n_heads;
    c->nkv = (int)h->n_kv_heads;
    c->hd = (int)h->head_dim;
    c->rot = (int)h->rot_dim;
    c->nk = (int)h->lin_k_heads;
    c->nv = (int)h->lin_v_heads;
    c->dk = (int)h->lin_k_dim;
    c->dv = (int)h->lin_v_dim;
    c->K = (int)h->conv_k;
    c->kd = c->nk * c->dk;
    c->vd = c->nv * c->dv;
    c->C = 2 * c->kd + c->vd;
    c->eps = h->rms_eps;
    c->eos = (int)h->eos_id;
    c->has_mtp = h->has_mtp ? 1 : 0;
}

// Engine limits of this build (beyond the reference's own, pinfer.c:152-156).
int check_limits(const pinfer_ctx *c) {
    char b[256];
    if (c->dk != 128 || c->dv != 128) {
        snprintf(b, sizeof b, "lin_k_dim %d / lin_v_dim %d not supported (this build runs 128 x 128 DeltaNet heads)", c->dk, c->dv);
        set_err(b);
        return PINFER_E_FORMAT;
    }
    if (c->hd % 32 || c->hd > 1024 || c->hd % 16 || c->rot > c->hd) {
        snprintf(b, sizeof b, "head_dim %d not supported (multiple of 32, <= 1024)", c->hd);
        set_err(b);
        return PINFER_E_FORMAT;
    }
    if (c->H % 256 || c->ffn % 256 || c->vd % 256 || (c->nq * c->hd) % 256) {
        set_err("dimensions must be multiples of 256 (Q4K superblocks)");
        return PINFER_E_FORMAT;
    }
    return PINFER_OK;
}

int alloc_state(pinfer_ctx *c);

int alloc_and_upload(pinfer_ctx *c) {
    const PqFile &f = c->file;
    c->weights = std::make_shared<WeightStore>();
    int rc = upload_mat(c, f.embed, &c->embed);
    if (rc) return rc;
    if (f.hdr->tied_embeddings) c->head = c->embed;
    else if ((rc = upload_mat(c, f.head, &c->head))) return rc;
    if ((rc = upload_floats(c, f.norm, c->H, &c->norm))) return rc;

    // RoPE tables for every position, computed like pf_rope_tables (forward.c:19-32)
    const int h2 = c->rot / 2;
    std::vector<float> cs((size_t)c->max_ctx * std::max(h2, 1)), sn(cs.size());
    const float theta = f.hdr->rope_theta;
    for (int i = 0; i < h2; i++) {
        const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)c->rot);
        for (int p = 0; p < c->max_ctx; p++) {
            const float ang = (float)p * inv;
            cs[(size_t)p * h2 + i] = cosf(ang);
            sn[(size_t)p * h2 + i] = sinf(ang);
        }
    }
    float *dcos, *dsin;
    if ((rc = upload_floats(c, cs.data(), cs.size(), &dcos))) return rc;
    if ((rc = upload_floats(c, sn.data(), sn.size(), &dsin))) return rc;

    const int cap = PINFER_SPEC_MAX_K + 1;
    c->lind = LinDims{c->C, c->K, c->kd, c->vd, c->nk, c->nv, c->nv / c->nk, c->dk, c->dv, cap,
                      c->C + c->vd + 2 * c->nv, c->eps};
    c->attd = AttnDims{c->nq, c->nkv, c->hd, c->rot, c->max_ctx, 2 * c->nq * c->hd + 2 * c->nkv * c->hd,
                       c->eps, dcos, dsin};
    c->attd.kv_dtype = c->kv_dtype;
    for (int l = 0; l < c->n_layers; l++) {
        const PqLayer &L = f.layers[l];
        auto &D = c->layers[l];
        D.is_full = L.is_full;
        if ((rc = upload_floats(c, L.in_norm, c->H, &D.in_norm))) return rc;
        if ((rc = upload_floats(c, L.post_norm, c->H, &D.post_norm))) return rc;
        if ((rc = upload_mat(c, L.gate, &D.gate)) || (rc = upload_mat(c, L.up, &D.up)) ||
            (rc = upload_mat(c, L.down, &D.down)))
            return rc;
        if (L.is_full) {
            const PqMat *parts[3] = {&L.q, &L.k, &L.v};
            if ((rc = upload_mats(c, parts, 3, &D.win)) || (rc = upload_mat(c, L.o, &D.out))) return rc;
            AttnLayer &A = c->att[l];
            float *qn, *kn;
            if ((rc = upload_floats(c, L.q_norm, c->hd, &qn)) || (rc = upload_floats(c, L.k_norm, c->hd, &kn))) return rc;
            A.q_norm = qn;
            A.k_norm = kn;
        } else {
            const PqMat *parts[4] = {&L.qkv, &L.z, &L.b, &L.a};
            if ((rc = upload_mats(c, parts, 4, &D.win)) || (rc = upload_mat(c, L.out, &D.out))) return rc;
            LinLayer &N = c->lin[c->n_lin];
            D.lin = c->n_lin++;
            std::vector<float> A(c->nv);   // A = -expf(A_log) (forward_lin.c:291), glibc on the host
            for (int h = 0; h < c->nv; h++) A[h] = L.A ? L.A[h] : -expf(L.A_log[h]);
            float *cw, *dA, *dt, *nw;
            if ((rc = upload_floats(c, L.conv_w, (size_t)c->C * c->K, &cw)) ||
                (rc = upload_floats(c, A.data(), c->nv, &dA)) ||
                (rc = upload_floats(c, L.dt_bias, c->nv, &dt)) ||
                (rc = upload_floats(c, L.lin_norm, c->dv, &nw)))
                return rc;
            N.conv_w = cw;
            N.A = dA;
            N.dt_bias = dt;
            N.norm_w = nw;
        }
    }
    if (f.hdr->has_mtp && f.mtp.ok) {   // the MTP head (mtp.c:8-32)
        const PqMtp &M = f.mtp;
        auto &D = c->mtp_layer;
        D.is_full = 1;
        const PqMat *parts[3] = {&M.layer.q, &M.layer.k, &M.layer.v};
        float *qn, *kn;
        if ((rc = upload_mat(c, M.fc, &c->mtp_fc)) ||
            (rc = upload_floats(c, M.norm_emb, c->H, &c->mtp_norm_emb)) ||
            (rc = upload_floats(c, M.norm_hid, c->H, &c->mtp_norm_hid)) ||
            (rc = upload_floats(c, M.norm_out, c->H, &c->mtp_norm_out)) ||
            (rc = upload_floats(c, M.layer.in_norm, c->H, &D.in_norm)) ||
            (rc = upload_floats(c, M.layer.post_norm, c->H, &D.post_norm)) ||
            (rc = upload_mat(c, M.layer.gate, &D.gate)) || (rc = upload_mat(c, M.layer.up, &D.up)) ||
            (rc = upload_mat(c, M.layer.down, &D.down)) || (rc = upload_mats(c, parts, 3, &D.win)) ||
            (rc = upload_mat(c, M.layer.o, &D.out)) || (rc = upload_floats(c, M.layer.q_norm, c->hd, &qn)) ||
            (rc = upload_floats(c, M.layer.k_norm, c->hd, &kn)))
            return rc;
        c->mtp_att.q_norm = qn;
        c->mtp_att.k_norm = kn;
        c->mtp_ok = true;
    }
    return alloc_state(c);
}

// This context's own buffers: recurrent and conv states, logs, KV caches, activations, the step
// block (everything but the model's parameters).
// int8 KV storage: the row scales beside a cache (the state blob carries them)
int alloc_kv_scales(pinfer_ctx *c, AttnLayer *A) {
    A->ks = A->vs = nullptr;
    if (c->kv_dtype != PINFER_KV_I8) return PINFER_OK;
    const size_t b = (size_t)c->nkv * c->max_ctx * sizeof(float);
    int rc;
    if ((rc = c->dalloc(&A->ks, b)) || (rc = c->dalloc(&A->vs, b))) return rc;
    return PINFER_OK;
}

int alloc_state(pinfer_ctx *c) {
    int rc;
    const int cap = PINFER_SPEC_MAX_K + 1;
    for (int l = 0; l < c->n_layers; l++) {
        const auto &D = c->layers[l];
        if (D.is_full) {
            AttnLayer &A = c->att[l];
            const size_t kv = (size_t)c->nkv * c->max_ctx * c->hd * sizeof(float);
            if ((rc = c->dalloc(&A.kc, kv)) || (rc = c->dalloc(&A.vc, kv))) return rc;
            if ((rc = alloc_kv_scales(c, &A))) return rc;
        } else {
            LinLayer &N = c->lin[D.lin];
            if ((rc = c->dalloc(&N.conv_state, sizeof(float) * (size_t)std::max(c->K - 1, 1) * c->C)) ||
                (rc = c->dalloc(&N.rec, sizeof(float) * (size_t)c->nv * c->dk * c->dv)) ||
                (rc = c->dalloc(&N.xin, sizeof(float) * (size_t)cap * c->C)) ||
                (rc = c->dalloc(&N.upd, sizeof(float) * 2 * (size_t)cap * c->nv * (c->dk + c->dv + 1))))
                return rc;
        }
    }
    if (c->mtp_ok) {
        const size_t kv = (size_t)c->nkv * c->max_ctx * c->hd * sizeof(float);
        if ((rc = alloc_kv_scales(c, &c->mtp_att))) return rc;
        if ((rc = c->dalloc(&c->mtp_att.kc, kv)) || (rc = c->dalloc(&c->mtp_att.vc, kv)) ||
            (rc = c->dalloc(&c->hn, sizeof(float) * kMaxRows * c->H)) ||
            (rc = c->dalloc(&c->mrows, sizeof(float) * kMaxRows * c->H)) ||
            (rc = c->dalloc(&c->mcur, sizeof(float) * c->H)) ||
            (rc = c->dalloc(&c->act_cat.q, (size_t)kMaxRows * 2 * c->H)) ||
            (rc = c->dalloc(&c->act_cat.d, sizeof(float) * kMaxRows * (2 * c->H / 32))) ||
            (rc = c->dalloc(&c->act_cat.fs, sizeof(float) * kMaxRows * (2 * c->H / 32))) ||
            (rc = c->dalloc(&c->msteps, sizeof(Step) * (PINFER_SPEC_MAX_K + 1))))
            return rc;
        c->act_cat.cols = 2 * c->H;
    }
    // activations
    const int ldy = std::max(c->lind.ldy, c->attd.ldy);
    const int mid = std::max(std::max(c->vd, c->nq * c->hd), c->ffn);
    if ((rc = c->dalloc(&c->x, sizeof(float) * kMaxRows * c->H)) ||
        (rc = c->dalloc(&c->y, sizeof(float) * kMaxRows * ldy)) ||
        (rc = c->dalloc(&c->qbuf, sizeof(float) * kMaxRows * c->nq * c->hd)) ||
        (rc = c->dalloc(&c->logits, sizeof(float) * kMaxRows * (size_t)c->vocab)) ||
        (rc = c->dalloc(&c->act_h.q, (size_t)kMaxRows * c->H)) ||
        (rc = c->dalloc(&c->act_h.d, sizeof(float) * kMaxRows * (c->H / 32))) ||
        (rc = c->dalloc(&c->act_h.fs, sizeof(float) * kMaxRows * (c->H / 32))) ||
        (rc = c->dalloc(&c->act_mid.q, (size_t)kMaxRows * mid)) ||
        (rc = c->dalloc(&c->act_mid.d, sizeof(float) * kMaxRows * (mid / 32))) ||
        (rc = c->dalloc(&c->act_mid.fs, sizeof(float) * kMaxRows * (mid / 32))) ||
        (rc = c->dalloc(&c->partial, sizeof(unsigned long long) * kMaxRows * c->head.npanels)) ||
        (rc = c->dalloc(&c->nan0, sizeof(int) * kMaxRows)) || (rc = c->dalloc(&c->step, sizeof(Step))) ||
        (rc = c->dalloc(&c->head_best, sizeof(unsigned long long) * kHeadFuseSlots)) ||
        (rc = c->dalloc(&c->head_ctr, sizeof(int))))
        return rc;
    c->act_h.cols = c->H;
    // prompt-lookup history and index (ngram.c pf_ngram_init: capacity max_ctx + 1, tables of
    // 2^bits entries, 2^bits >= 2 x capacity, 10 <= bits <= 24)
    c->ng_cap = c->max_ctx + 1;
    c->ng_bits = 10;
    while (c->ng_bits < 24 && (1 << c->ng_bits) < 2 * c->ng_cap) c->ng_bits++;
    if ((rc = c->dalloc(&c->ng_hist, sizeof(int) * (size_t)c->ng_cap)) ||
        (rc = c->dalloc(&c->ng_tab, sizeof(int) * ((size_t)3 << c->ng_bits))))
        return rc;
    {
        const int dims[2] = {c->ng_cap, c->ng_bits};
        int *const ptrs[2] = {c->ng_hist, c->ng_tab};
        static_assert(offsetof(Step, ng_bits) == offsetof(Step, hist_cap) + sizeof(int), "adjacent fields");
        static_assert(offsetof(Step, ng_tab) == offsetof(Step, hist) + sizeof(int *), "adjacent fields");
        CUDA_OK(cudaMemcpy(&c->step->hist_cap, dims, sizeof dims, cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(&c->step->hist, ptrs, sizeof ptrs, cudaMemcpyHostToDevice));
    }
    CUDA_OK(cudaMallocHost(&c->h_step, sizeof(Step)));
    memset(c->h_step, 0, sizeof(Step));

    if (kernels_init(c->max_ctx, c->hd, c->lind.rep) != 0) return PINFER_E_NOMEM;
    return PINFER_OK;
}

Act mid_act(pinfer_ctx *c, int cols) {
    Act a = c->act_mid;
    a.cols = cols;
    return a;
}

// One forward pass over the rows described by the Step block (<= nmax rows).
// head: 0 none, 1 logits + argmax, 2 argmax only (no logits written)
// accept_follows: k_accept runs right after the pass (verify rounds); it sets the deferred
// commit itself, so the pass's own k_pass_end is left out.
void enqueue_forward(pinfer_ctx *c, int nmax, int head, bool export_normed = false, bool accept_follows = false) {
    cudaStream_t s = c->stream;
    launch_embed(c->embed, c->step, c->x, c->H, s);
    AttnDims ad = c->attd;
    ad.rps = std::min(nmax, kMaxRows);   // attention grids cover the pass's rows only
    for (int l = 0; l < c->n_layers; l++) {
        auto &D = c->layers[l];
        // the next layer's matrices into L2 while this layer runs, so the weight copies its
        // kernels issue before their griddepcontrol.wait are L2 hits
        L2Prefetch pf;
        if (l + 1 < c->n_layers) {
            const auto &N = c->layers[l + 1];
            for (const Mat *m : {&N.win, &N.out, &N.gate, &N.up, &N.down})
                pf.add(m->w, (size_t)m->npanels * m->nsb * kUnitBytes);
        }
        if (D.is_full) {
            // and this layer's K / V rows of the positions the pass attends to
            const size_t kvb = (size_t)ad.max_ctx * c->hd * sizeof(float);
            for (int g = 0; g < c->nkv; g++) {
                pf.add(c->att[l].kc + (size_t)g * ad.max_ctx * c->hd, kvb, (unsigned)(c->hd * sizeof(float)));
                pf.add(c->att[l].vc + (size_t)g * ad.max_ctx * c->hd, kvb, (unsigned)(c->hd * sizeof(float)));
            }
            const Act o = mid_act(c, c->nq * c->hd);
            launch_matvec_norm(D.win, c->x, D.in_norm, c->eps, c->step, c->y, c->attd.ldy, nmax, c->act_h, s, pf);
            launch_attn_prep(c->att[l], ad, c->y, c->qbuf, c->step, s);
            launch_attn(c->att[l], ad, c->y, c->qbuf, c->step, o, s);
            launch_matvec(D.out, o, c->step, c->x, c->H, 1, nmax, s);
        } else {
            const Act o = mid_act(c, c->vd);
            launch_matvec_norm(D.win, c->x, D.in_norm, c->eps, c->step, c->y, c->lind.ldy, nmax, c->act_h, s, pf);
            launch_deltanet(c->lin[D.lin], c->lind, c->y, c->step, o, s, 1, nmax);
            launch_matvec(D.out, o, c->step, c->x, c->H, 1, nmax, s);
        }
        const Act h = mid_act(c, c->ffn);
        launch_matvec_swiglu_norm(D.gate, D.up, c->x, D.post_norm, c->eps, c->step, h, nmax, c->act_h, s);
        launch_matvec(D.down, h, c->step, c->x, c->H, 1, nmax, s);
    }
    if (export_normed) launch_norm_rows(c->x, c->norm, c->H, c->eps, c->step, c->hn, s);   // pf_forward_h normed
    if (head) {
        // sharded: this GPU's vocabulary rows only, logits at their global columns
        const bool sharded = c->shard_world > 1;
        const Mat &HW = sharded ? c->head_view : c->head;
        float *lg = head == 1 ? c->logits + c->head_row0 : nullptr;
        if (nmax <= 4) {   // unsharded: the head kernel finishes the argmax itself
            launch_matvec_head_norm(HW, c->x, c->norm, c->eps, c->step, lg, c->vocab, c->partial, c->nan0,
                                    nmax, s, c->head_row0, sharded ? nullptr : c->head_best,
                                    sharded ? nullptr : c->head_ctr);
        } else {
            launch_norm_quant(c->x, c->norm, c->H, c->eps, c->step, c->act_h, s);
            launch_matvec_head(HW, c->act_h, c->step, lg, c->vocab, c->partial, c->nan0, nmax, s,
                               c->head_row0);
        }
        if (!sharded) {
            if (nmax > 4) launch_argmax_final(c->partial, c->nan0, c->head.npanels, c->step, s);
        } else {
            // one all-reduce (max) of the (value, first index) keys across the shards: the
            // tie and NaN rules of pf_argmax hold because the keys order exactly as they do
            const NcclApi *n = nccl_api(nullptr, 0);
            launch_argmax_keys(c->partial, c->nan0, HW.npanels, c->step, c->d_keys, s);
            n->all_reduce(c->d_keys, c->d_keys, 2 * kMaxRows, ncclUint64, ncclMax, c->nccl, s);
            launch_keys_argmax(c->d_keys, c->step, s);
            if (head == 1) {   // logits of every row for the API: in-place all-gather of the shards
                const size_t S = (size_t)c->head_view.rows;
                n->group_start();
                for (int v = 0; v < nmax; v++)
                    n->all_gather(c->logits + (size_t)v * c->vocab + c->head_row0, c->logits + (size_t)v * c->vocab,
                                  S, ncclFloat, c->nccl, s);
                n->group_end();
            }
        }
    }
    if (!accept_follows) launch_pass_end(c->step, s);
}

// One MTP pass (pf_mtp_forward, mtp.c:62-100) over the rows of step block ms: h [n][H] hidden
// rows, ms->tokens the tokens that follow them, positions ms->pos0..; writes the MTP KV rows,
// the normed outputs m (c->mrows) and, with head, the argmax over the draft vocabulary
// (ms->argmax). Uses the main pass's scratch buffers, so it runs between main passes.
void enqueue_mtp(pinfer_ctx *c, Step *ms, const float *h, int nmax, bool head, bool conf = false) {
    cudaStream_t s = c->stream;
    const auto &D = c->mtp_layer;
    launch_mtp_input(c->embed, h, ms, c->mtp_norm_emb, c->mtp_norm_hid, c->H, c->eps, c->act_cat, s);
    launch_matvec(c->mtp_fc, c->act_cat, ms, c->x, c->H, 0, nmax, s);   // u = fc [e | h]
    const Act o = mid_act(c, c->nq * c->hd);
    launch_matvec_norm(D.win, c->x, D.in_norm, c->eps, ms, c->y, c->attd.ldy, nmax, c->act_h, s);
    AttnDims ad = c->attd;
    ad.rps = std::min(nmax, kMaxRows);   // attention grids cover the pass's rows only
    launch_attn_prep(c->mtp_att, ad, c->y, c->qbuf, ms, s);
    launch_attn(c->mtp_att, ad, c->y, c->qbuf, ms, o, s);
    launch_matvec(D.out, o, ms, c->x, c->H, 1, nmax, s);
    const Act hm = mid_act(c, c->ffn);
    launch_matvec_swiglu_norm(D.gate, D.up, c->x, D.post_norm, c->eps, ms, hm, nmax, c->act_h, s);
    launch_matvec(D.down, hm, ms, c->x, c->H, 1, nmax, s);
    launch_norm_rows(c->x, c->mtp_norm_out, c->H, c->eps, ms, c->mrows, s);   // m = mtp.norm(u)
    if (head) {
        if (nmax <= 4) {   // the head kernel finishes the argmax itself
            launch_matvec_head_norm(c->mtp_head, c->x, c->mtp_norm_out, c->eps, ms, conf ? c->logits : nullptr, c->vocab,
                                    c->partial, c->nan0, nmax, s, 0, c->head_best, c->head_ctr);
        } else {
            launch_norm_quant(c->x, c->mtp_norm_out, c->H, c->eps, ms, c->act_h, s);
            launch_matvec_head(c->mtp_head, c->act_h, ms, conf ? c->logits : nullptr, c->vocab, c->partial, c->nan0,
                               nmax, s);
        }
        if (nmax > 4) launch_argmax_final(c->partial, c->nan0, c->mtp_head.npanels, ms, s);
        // adaptive: the top-1 probability of the pass's newest draft (its last row)
        if (conf) launch_conf(c->logits, c->vocab, c->mtp_head.rows, ms, c->step, s);
    }
}

// The head's first nv rows, the draft vocabulary (spec.c:88-91, mtp.c:92-97).
void set_mtp_head(pinfer_ctx *c, int nv) {
    c->mtp_head = c->head;
    c->mtp_head.rows = nv;
    c->mtp_head.npanels = (nv + kPanelRows - 1) / kPanelRows;
}

int sync(pinfer_ctx *c) {
    CUDA_OK(cudaStreamSynchronize(c->stream));
    return PINFER_OK;
}

int read_step(pinfer_ctx *c) {
    CUDA_OK(cudaMemcpyAsync(c->h_step, c->step, sizeof(Step), cudaMemcpyDeviceToHost, c->stream));
    return sync(c);
}

int flush_pending(pinfer_ctx *c) {
    launch_flush(c->lin, c->n_lin, c->lind, c->step, c->stream);
    return PINFER_OK;
}

// Feed tokens through the model (pf_forward_h, forward.c:149-165: the rows of a chunk give the
// same results whatever the chunk size). The rows before the last pass go through the tensor-
// core GEMMs in chunks of up to kPrefillRows when there are more than one pass's worth of them;
// the last (n - 1) % kMaxRows + 1 rows, whose logits or argmax are wanted, take one CUDA-core
// pass. want: 0 nothing, 1 logits + argmax of the last pass, 2 argmax only.
int forward_tokens(pinfer_ctx *c, const int32_t *tokens, int n, int want) {
    const int tail = want ? (n - 1) % kMaxRows + 1 : 0;
    if (n - tail > kMaxRows && prefill_gemm_ok(c)) {
        const int rc = prefill_gemm(c, tokens, n - tail, nullptr);
        if (rc) return rc;
        tokens += n - tail;
        n = tail;
    }
    for (int t0 = 0; t0 < n; t0 += kMaxRows) {
        const int nb = std::min(kMaxRows, n - t0);
        const bool last = t0 + nb == n;
        launch_set_pass(c->step, nb, c->n_past, 0, tokens + t0, c->stream);
        enqueue_forward(c, kMaxRows, last ? want : 0);
        c->n_past += nb;
    }
    CUDA_OK(cudaGetLastError());
    return PINFER_OK;
}

int validate_tokens(const pinfer_ctx *c, const int32_t *tokens, int n) {
    if (!c || !tokens || n <= 0) return PINFER_E_ARG;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c->vocab) return PINFER_E_ARG;
    if (n > c->max_ctx - c->n_past) return PINFER_E_CTX_FULL;
    return PINFER_OK;
}

void drop_graphs(pinfer_ctx *c);

// Output and target-token buffers of a generation of n_max tokens. Captured round graphs hold
// the buffers' addresses, so growing them drops the graphs (recaptured on next use); they grow
// at least twofold to keep that rare.
int ensure_out(pinfer_ctx *c, int n_max) {
    if (c->out_cap >= n_max) return PINFER_OK;
    const int cap = std::max(n_max, std::max(2 * c->out_cap, 256));
    CUDA_OK(cudaStreamSynchronize(c->stream));   // no round in flight uses the old buffers
    drop_graphs(c);
    cudaFree(c->d_out);
    cudaFree(c->d_greedy);
    c->d_out = nullptr;
    c->d_greedy = nullptr;
    c->out_cap = 0;
    CUDA_OK(cudaMalloc(&c->d_out, sizeof(int) * (size_t)cap));
    CUDA_OK(cudaMalloc(&c->d_greedy, sizeof(int) * (size_t)cap));
    CUDA_OK(cudaMemset(c->d_greedy, 0, sizeof(int) * (size_t)cap));
    c->out_cap = cap;
    return PINFER_OK;
}

// The graph of one round at draft depth k (drafter 0: synthetic drafts or none, 1: the MTP
// head) with n-gram drafts of up to `ngram` tokens: the verify pass holds max(k, ngram) + 1 rows.
int round_graph(pinfer_ctx *c, int k, cudaGraphExec_t *out, int drafter = 0, int nv = 0, int ngram = 0,
                int adaptive = 0) {
    if (drafter == 1 && c->round_graph_mtp[k] &&
        (c->graph_nv[k] != nv || c->graph_ng[k] != ngram || c->graph_ad[k] != adaptive)) {
        cudaGraphExecDestroy(c->round_graph_mtp[k]);
        c->round_graph_mtp[k] = nullptr;
    }
    if (drafter == 0 && ngram > 0 && c->round_graph_ng[ngram] && c->graph_ng_ad[ngram] != adaptive) {
        cudaGraphExecDestroy(c->round_graph_ng[ngram]);
        c->round_graph_ng[ngram] = nullptr;
    }
    cudaGraphExec_t &slot = drafter == 1 ? c->round_graph_mtp[k]
                                         : (ngram > 0 ? c->round_graph_ng[ngram] : c->round_graph[k]);
    if (slot) {
        *out = slot;
        return PINFER_OK;
    }
    const int rows = std::max(k, ngram) + 1;
    const int nmax = rows <= 1 ? 1 : rows <= 4 ? 4 : rows <= 8 ? 8 : 16;
    cudaStream_t s = c->stream;
    cudaGraph_t g;
    CUDA_OK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    if (drafter == 1) {
        // pf_spec_decode with MTP drafts (spec.c:300-374): the chain drafts 2..ke, the verify
        // pass (with its normed rows), acceptance, then the MTP pass over the committed rows,
        // which drafts the next round's first token
        // adaptive (spec_adapt.c): timestamps of the round's phases, and the top-1 probability
        // of every MTP draft for the chain rule
        set_mtp_head(c, nv);
        if (adaptive) launch_stamp(c->step, 0, s);
        for (int i = 1; i < k; i++) {
            launch_mtp_chain_set(c->step, c->msteps + i, i, s);
            enqueue_mtp(c, c->msteps + i, c->mcur, 1, true, adaptive != 0);
            launch_mtp_chain_take(c->step, c->msteps + i, i, c->mrows, c->mcur, c->H, s);
        }
        if (adaptive) launch_stamp(c->step, 1, s);
        enqueue_forward(c, nmax, 2, true, !adaptive);
        if (adaptive) launch_stamp(c->step, 2, s);
        launch_accept(c->step, c->d_greedy, c->d_out, s);
        launch_mtp_pending_set(c->step, c->msteps, s);
        enqueue_mtp(c, c->msteps, c->hn, nmax, true, adaptive != 0);
        launch_mtp_pending_take(c->step, c->msteps, c->mrows, c->mcur, c->H, s);
    } else {
        if (adaptive) {
            launch_stamp(c->step, 0, s);
            launch_stamp(c->step, 1, s);
        }
        enqueue_forward(c, nmax, 2, false, !adaptive);
        if (adaptive) launch_stamp(c->step, 2, s);
        launch_accept(c->step, c->d_greedy, c->d_out, s);
    }
    CUDA_OK(cudaStreamEndCapture(s, &g));
    cudaGraphExec_t ex;
    CUDA_OK(cudaGraphInstantiate(&ex, g, 0));
    cudaGraphDestroy(g);
    slot = ex;
    if (drafter == 1) {
        c->graph_nv[k] = nv;
        c->graph_ng[k] = ngram;
        c->graph_ad[k] = adaptive;
    }
    if (drafter == 0 && ngram > 0) c->graph_ng_ad[ngram] = adaptive;
    if (drafter == 0 && ngram == 0) c->round_nmax[k] = nmax;
    *out = ex;
    return PINFER_OK;
}

void drop_graphs(pinfer_ctx *c) {
    for (auto &g : c->round_graph)
        if (g) { cudaGraphExecDestroy(g); g = nullptr; }
    for (auto &g : c->round_graph_mtp)
        if (g) { cudaGraphExecDestroy(g); g = nullptr; }
    for (auto &g : c->round_graph_ng)
        if (g) { cudaGraphExecDestroy(g); g = nullptr; }
}

// Zero MTP KV rows [from, to) of every group (spec.c:166-170: positions consumed without the
// MTP head hold no MTP rows, and drafts must not attend to stale memory).
int zero_mtp_rows(pinfer_ctx *c, int from, int to) {
    if (!c->mtp_ok || to <= from) return PINFER_OK;
    const size_t row = (size_t)c->hd * sizeof(float), gstride = (size_t)c->max_ctx * c->hd;
    for (int g = 0; g < c->nkv; g++) {
        CUDA_OK(cudaMemsetAsync(c->mtp_att.kc + g * gstride + (size_t)from * c->hd, 0, (size_t)(to - from) * row, c->stream));
        CUDA_OK(cudaMemsetAsync(c->mtp_att.vc + g * gstride + (size_t)from * c->hd, 0, (size_t)(to - from) * row, c->stream));
        if (c->mtp_att.ks) {   // int8 storage: the rows' scales too (forward_kv.c:127-137)
            const size_t sc = (size_t)g * c->max_ctx + from, n = (size_t)(to - from) * sizeof(float);
            CUDA_OK(cudaMemsetAsync(c->mtp_att.ks + sc, 0, n, c->stream));
            CUDA_OK(cudaMemsetAsync(c->mtp_att.vs + sc, 0, n, c->stream));
        }
    }
    return PINFER_OK;
}

// The prompt with the MTP head (pf_spec_prefill, spec.c:172-195): chunk by chunk the main pass
// with its normed rows, then the MTP pass over the same rows (row i with token i + 1; the last
// row with the first generated token), which fills the MTP KV rows and drafts d1. The rows
// before the last pass go through the GEMM chunks (nb_prefill.cu), the last pass as 16 rows.
int forward_tokens_mtp(pinfer_ctx *c, const int32_t *tokens, int n) {
    int rc;
    if ((rc = zero_mtp_rows(c, c->mtp_rows, c->n_past))) return rc;
    // the rows before the last pass: GEMM chunks with the MTP pass over each (every such row's
    // next token is in the prompt)
    const int tail = (n - 1) % kMaxRows + 1;
    if (n - tail > kMaxRows && prefill_gemm_ok(c)) {
        if ((rc = prefill_gemm(c, tokens, n - tail, nullptr, tokens + 1))) return rc;
        tokens += n - tail;
        n = tail;
    }
    int next[kMaxRows];
    for (int t0 = 0; t0 < n; t0 += kMaxRows) {
        const int nb = std::min(kMaxRows, n - t0);
        const bool last = t0 + nb == n;
        launch_set_pass(c->step, nb, c->n_past, 0, tokens + t0, c->stream);
        enqueue_forward(c, kMaxRows, last ? 2 : 0, true);
        for (int i = 0; i < nb; i++) next[i] = t0 + i + 1 < n ? tokens[t0 + i + 1] : 0;
        launch_set_pass(c->msteps, nb, c->n_past, 0, next, c->stream);
        if (last) launch_mtp_prefill_fix(c->step, c->msteps, c->stream);
        enqueue_mtp(c, c->msteps, c->hn, kMaxRows, last);
        if (last) launch_mtp_pending_take(c->step, c->msteps, c->mrows, c->mcur, c->H, c->stream);
        c->n_past += nb;
    }
    c->mtp_rows = c->n_past;
    CUDA_OK(cudaGetLastError());
    return PINFER_OK;
}

struct GenRequest {
    const int32_t *prompt;
    int n_prompt;
    int32_t *out;
    int n_max;
    int k;                    // drafts per round (0 = plain greedy)
    const int32_t *greedy;    // synthetic drafter's target stream (k > 0), n_max entries
    unsigned long long seed;
    unsigned p24;
    const pinfer_gen_opts *opts;
    int append;
    long long stats[3];
    float decode_ms;          // device time of the round loop (events on the context's stream)
    int drafter = 0;          // 0 synthetic drafts, 1 the MTP head
    int nv = 0;               // MTP draft vocabulary
    int ngram = 0;            // longest n-gram (prompt-lookup) draft, 0 = none
    int adaptive = 0;         // the adaptive speculation policy
    long long ng_stats[3] = {0, 0, 0};
};

// The n-gram history before a prompt is fed (pf_spec_prefill, spec.c:163-171): the fed tokens
// plus the last emitted one, which a continuation prompt leads with, so a continuation drops
// that token and appends the prompt; any other context (a fresh start, pinfer_eval, a loaded
// state) is not described by the history, which starts anew with the prompt.
int ngram_prefill(pinfer_ctx *c, const int32_t *prompt, int n, int append, int base) {
    if (!c->ng_hist) return PINFER_OK;
    if (append && c->ng_n == base + 1) {
        c->ng_n--;
        c->ng_idx = std::min(c->ng_idx, c->ng_n);   // stale entries fail the checks
    } else {
        c->ng_n = c->ng_idx = 0;
        CUDA_OK(cudaMemsetAsync(c->ng_tab, 0, sizeof(int) * ((size_t)3 << c->ng_bits), c->stream));
    }
    const int m = std::min(n, c->ng_cap - c->ng_n);
    if (m > 0) {
        CUDA_OK(cudaMemcpyAsync(c->ng_hist + c->ng_n, prompt, sizeof(int) * (size_t)m, cudaMemcpyHostToDevice,
                                c->stream));
        c->ng_n += m;
    }
    const int v[2] = {c->ng_n, c->ng_idx};
    static_assert(offsetof(Step, hist_idx) == offsetof(Step, hist_n) + sizeof(int), "adjacent fields");
    CUDA_OK(cudaMemcpyAsync(&c->step->hist_n, v, sizeof v, cudaMemcpyHostToDevice, c->stream));
    return sync(c);   // v lives on this stack frame
}

// Generation (generate / pf_spec_prefill / pf_spec_decode, spec.c:153-416): prefill, then
// rounds of [verify pass, argmax, greedy acceptance, commit, next drafts] replayed from one
// CUDA graph with no host round trip until enough tokens can have been produced; finally the
// deferred commit is applied (pf_lin_flush).
int generate_impl(pinfer_ctx *c, GenRequest *r, int *status) {
    int dummy;
    if (!status) status = &dummy;
    *status = PINFER_OK;
    if (!c || !r->out || r->n_max <= 0 || r->k < 0 || r->k > PINFER_SPEC_MAX_K ||
        (r->opts && r->opts->n_stop > 0 && !r->opts->stop_ids) || !r->prompt || r->n_prompt <= 0)
        return *status = PINFER_E_ARG;
    if (!r->append) pinfer_reset(c);
    int rc = validate_tokens(c, r->prompt, r->n_prompt);
    if (rc) return *status = rc;
    if ((rc = ensure_out(c, r->n_max))) return *status = rc;
    if (r->k > 0 && r->greedy)
        CUDA_OK(cudaMemcpyAsync(c->d_greedy, r->greedy, sizeof(int) * r->n_max, cudaMemcpyHostToDevice, c->stream));
    const bool host_loop = r->opts && (r->opts->on_token || r->opts->n_stop > 8);
    GenArgs g{};
    g.n_max = r->n_max;
    g.k = r->k;
    g.eos = c->eos;
    g.n_stop = host_loop || !r->opts ? 0 : r->opts->n_stop;
    for (int i = 0; i < g.n_stop; i++) g.stop_ids[i] = r->opts->stop_ids[i];
    g.max_ctx = c->max_ctx;
    g.vocab = c->vocab;
    g.p24 = r->p24;
    g.seed = r->seed;
    g.drafter = r->drafter;
    g.ngram = r->ngram;
    g.adaptive = r->adaptive;
    if (host_loop) g.eos = -1;   // the host decides when to stop (one token per round)
    if ((rc = ngram_prefill(c, r->prompt, r->n_prompt, r->append, c->n_past))) return *status = rc;
    launch_set_gen(c->step, g, c->stream);
    if (r->drafter == 1) {
        set_mtp_head(c, r->nv);
        if ((rc = forward_tokens_mtp(c, r->prompt, r->n_prompt))) return *status = rc;
    } else if ((rc = forward_tokens(c, r->prompt, r->n_prompt, 2))) {
        return *status = rc;
    }
    launch_gen_start(c->step, c->d_greedy, c->d_out, c->stream);
    cudaGraphExec_t ex;
    if ((rc = round_graph(c, r->k, &ex, r->drafter, r->nv, r->ngram, r->adaptive))) return *status = rc;
    int count = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cudaEventCreate(&ev0);
    cudaEventCreate(&ev1);
    cudaEventRecord(ev0, c->stream);
    if (!host_loop) {
        if ((rc = read_step(c))) return *status = rc;
        while (!c->h_step->done) {
            const int left = r->n_max - c->h_step->count;
            const int reps = std::max(1, (left + r->k) / (r->k + 1));
            for (int i = 0; i < reps; i++) CUDA_OK(cudaGraphLaunch(ex, c->stream));
            if ((rc = read_step(c))) return *status = rc;
        }
        cudaEventRecord(ev1, c->stream);
        count = c->h_step->count;
        CUDA_OK(cudaMemcpy(r->out, c->d_out, sizeof(int) * count, cudaMemcpyDeviceToHost));
    } else {
        // tokens reach the callback one by one as soon as they are final (pinfer.h:122-124)
        int seen = 0, stop = 0;
        for (;;) {
            if ((rc = read_step(c))) return *status = rc;
            const int have = c->h_step->count;
            std::vector<int> buf(have - seen);
            if (have > seen)
                CUDA_OK(cudaMemcpy(buf.data(), c->d_out + seen, sizeof(int) * (have - seen), cudaMemcpyDeviceToHost));
            for (int i = 0; i < have - seen && !stop; i++) {
                const int tok = buf[i];
                r->out[count++] = tok;
                stop = count >= r->n_max;
                if (r->opts->on_token && r->opts->on_token(tok, r->opts->user)) stop = 1;
                if (tok == c->eos) stop = 1;
                for (int j = 0; j < r->opts->n_stop && !stop; j++) stop = tok == r->opts->stop_ids[j];
            }
            seen = have;
            if (stop || c->h_step->done) break;
            CUDA_OK(cudaGraphLaunch(ex, c->stream));
        }
        cudaEventRecord(ev1, c->stream);
    }
    cudaEventSynchronize(ev1);
    cudaEventElapsedTime(&r->decode_ms, ev0, ev1);
    cudaEventDestroy(ev0);
    cudaEventDestroy(ev1);
    if ((rc = read_step(c))) return *status = rc;
    r->stats[0] = c->h_step->rounds;
    r->stats[1] = c->h_step->drafted;
    r->stats[2] = c->h_step->accepted;
    r->ng_stats[0] = c->h_step->ng_rounds;
    r->ng_stats[1] = c->h_step->ng_drafted;
    r->ng_stats[2] = c->h_step->ng_accepted;
    c->ng_n = c->h_step->hist_n;
    c->ng_idx = c->h_step->hist_idx;
    *status = c->h_step->status;
    c->n_past = c->h_step->pos0;
    if (r->drafter == 1) c->mtp_rows = c->n_past;   // every committed row had its MTP pass
    flush_pending(c);
    if ((rc = sync(c))) return *status = rc;
    return count;
}

}  // namespace

// ================================================================ public C API
extern "C" {

pinfer_params pinfer_default_params(void) {
    pinfer_params p = {4, 4096, PINFER_KV_F32, 0.0f};
    return p;
}

const char *pinfer_version(void) { return "0.3.0"; }

pinfer_ctx *pinfer_load(const char *path, const pinfer_params *params, int *err) {
    pinfer_params p = params ? *params : pinfer_default_params();
    if (p.n_threads <= 0) p.n_threads = 4;
    if (p.max_ctx <= 0) p.max_ctx = 4096;
    int rc = PINFER_OK;
    pinfer_ctx *c = nullptr;
    int ndev = 0;
    if (!path) rc = PINFER_E_ARG;
    else if (!std::isfinite(p.gpu_split) || p.gpu_split < 0.0f || p.gpu_split > 1.0f) {
        set_err("gpu_split must be finite and in [0,1]");
        rc = PINFER_E_ARG;
    } else if (p.kv_dtype < PINFER_KV_F32 || p.kv_dtype > PINFER_KV_I8) {
        set_err("unknown kv_dtype");
        rc = PINFER_E_ARG;
    } else if (p.max_ctx > 1 << 20) {
        set_err("max_ctx too large");
        rc = PINFER_E_ARG;
    } else {
        c = new (std::nothrow) pinfer_ctx();
        if (!c) rc = PINFER_E_NOMEM;
    }
    if (c) {
        // the file is validated first (model.c order), then the device is required
        rc = c->file.open_file(path);
        if (rc == PINFER_OK) {
            c->kv_dtype = p.kv_dtype;
            set_dims(c);
            c->max_ctx = p.max_ctx;
            c->fp = c->file.fingerprint();
            rc = check_limits(c);
        }
        if (rc == PINFER_OK && (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1)) {
            set_err("no CUDA device: this library runs on an NVIDIA B200 and has no CPU path");
            rc = PINFER_E_NOMEM;
        }
        if (rc == PINFER_OK) cudaGetDevice(&c->device);
        if (rc == PINFER_OK && cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
            set_err("cannot create a CUDA stream");
            rc = PINFER_E_NOMEM;
        }
        if (rc == PINFER_OK) rc = alloc_and_upload(c);
        if (rc == PINFER_OK) {
            c->hdr = *c->file.hdr;
            c->file.close_file();   // everything lives in HBM now
            if (cudaDeviceSynchronize() != cudaSuccess) rc = PINFER_E_NOMEM;
        }
    }
    if (rc != PINFER_OK) {
        pinfer_free(c);
        c = nullptr;
    }
    if (err) *err = rc;
    return c;
}

void pinfer_free(pinfer_ctx *c) {
    if (!c) return;
    if (c->stream) cudaStreamSynchronize(c->stream);
    drop_graphs(c);
    if (c->nccl) {
        const NcclApi *n = nccl_api(nullptr, 0);
        if (n) n->comm_destroy(c->nccl);
    }
    for (void *p : c->allocs) cudaFree(p);
    cudaFree(c->d_out);
    cudaFree(c->d_greedy);
    cudaFree(c->ck_buf);
    if (c->h_step) cudaFreeHost(c->h_step);
    if (c->stream) cudaStreamDestroy(c->stream);
    c->file.close_file();
    delete c;
}

void pinfer_reset(pinfer_ctx *c) {
    if (!c) return;
    for (int i = 0; i < c->n_lin; i++) {
        cudaMemsetAsync(c->lin[i].conv_state, 0, sizeof(float) * (size_t)std::max(c->K - 1, 1) * c->C, c->stream);
        cudaMemsetAsync(c->lin[i].rec, 0, sizeof(float) * (size_t)c->nv * c->dk * c->dv, c->stream);
    }
    launch_flush(nullptr, 0, c->lind, c->step, c->stream);   // clears any owed commit
    c->n_past = 0;
    c->mtp_rows = 0;
    c->ck_valid = 0;
}

int pinfer_eval(pinfer_ctx *c, const int32_t *tokens, int n, float *logits) {
    int rc = validate_tokens(c, tokens, n);
    if (rc) return rc;
    if ((rc = forward_tokens(c, tokens, n, logits ? 1 : 0))) return rc;
    if (logits) {
        const int last = (n - 1) % kMaxRows;
        CUDA_OK(cudaMemcpyAsync(logits, c->logits + (size_t)last * c->vocab, sizeof(float) * c->vocab,
                                cudaMemcpyDeviceToHost, c->stream));
    }
    return sync(c);
}

int pinfer_eval_select(pinfer_ctx *c, const int32_t *tokens, int n, const int32_t *ids, int n_ids,
                       float *out) {
    if (!c || n_ids < 0 || (n_ids > 0 && (!ids || !out))) return PINFER_E_ARG;
    for (int i = 0; i < n_ids; i++)
        if (ids[i] < 0 || ids[i] >= c->vocab) return PINFER_E_ARG;
    int rc = validate_tokens(c, tokens, n);
    if (rc) return rc;
    if ((rc = forward_tokens(c, tokens, n, n_ids > 0 ? 1 : 0))) return rc;
    if ((rc = sync(c))) return rc;
    if (n_ids == 0) return PINFER_OK;
    const int last = (n - 1) % kMaxRows;
    for (int i = 0; i < n_ids; i++)
        CUDA_OK(cudaMemcpy(out + i, c->logits + (size_t)last * c->vocab + ids[i], sizeof(float),
                           cudaMemcpyDeviceToHost));
    return PINFER_OK;
}

pinfer_spec_params pinfer_default_spec_params(void) {
    pinfer_spec_params p = {4, 32768, 1, 7};
    return p;
}

int pinfer_has_mtp(const pinfer_ctx *c) { return c && c->has_mtp ? 1 : 0; }

static int generate_api(pinfer_ctx *c, const int32_t *prompt, int n_prompt, int32_t *out,
                        int n_max, const pinfer_spec_params *sp, const pinfer_gen_opts *opts,
                        pinfer_spec_stats *stats, int *status, int append) {
    int dummy;
    if (!status) status = &dummy;
    if (sp && (sp->k < 0 || sp->k > PINFER_SPEC_MAX_K || sp->ngram < 0 || sp->ngram > PINFER_SPEC_MAX_K))
        return *status = PINFER_E_ARG;
    if (sp && sp->k > 0 && c && !(c->has_mtp && c->mtp_ok)) return *status = PINFER_E_FORMAT;
    // k > 0: drafts from the MTP head, k per round (pf_spec_decode); ngram > 0: prompt-lookup
    // drafts of up to ngram tokens where the history's tail occurred before (with or without the
    // MTP head); adaptive: k becomes an upper bound (the chain runs while the newest draft's
    // top-1 probability is >= 0.6) and plain steps replace speculation while it measures slower
    // (spec_adapt.c). The tokens never depend on any of this (pinfer.h:70-73).
    GenRequest r{prompt, n_prompt, out, n_max, 0, nullptr, 0, 0, opts, append, {0, 0, 0}, 0.0f};
    if (sp && sp->k > 0) {
        r.k = sp->k;
        r.drafter = 1;
        const int v = sp->draft_vocab;   // spec.c:88-91
        r.nv = v >= 4 && v < c->vocab ? (v & ~3) : c->vocab;
    }
    if (sp) {
        r.ngram = sp->ngram;
        r.adaptive = (r.k > 0 || r.ngram > 0) && sp->adaptive ? 1 : 0;
    }
    const int n = generate_impl(c, &r, status);
    if (stats && n >= 0 && (r.k > 0 || r.ngram > 0)) {   // accumulated, never reset (pinfer.h:110-116)
        stats->rounds += r.stats[0];
        stats->drafted += r.stats[1];
        stats->accepted += r.stats[2];
        stats->ngram_rounds += r.ng_stats[0];
        stats->ngram_drafted += r.ng_stats[1];
        stats->ngram_accepted += r.ng_stats[2];
    }
    return n;
}

int pinfer_generate_greedy_ex(pinfer_ctx *c, const int32_t *prompt, int n_prompt, int32_t *out,
                              int n_max, const pinfer_spec_params *sp, const pinfer_gen_opts *opts,
                              pinfer_spec_stats *stats, int *status) {
    return generate_api(c, prompt, n_prompt, out, n_max, sp, opts, stats, status, 0);
}

int pinfer_generate_greedy_cont(pinfer_ctx *c, const int32_t *prompt, int n_prompt, int32_t *out,
                                int n_max, const pinfer_spec_params *sp, const pinfer_gen_opts *opts,
                                pinfer_spec_stats *stats, int *status) {
    return generate_api(c, prompt, n_prompt, out, n_max, sp, opts, stats, status, 1);
}

int pinfer_generate_greedy(pinfer_ctx *c, const int32_t *prompt, int n_prompt, int32_t *out,
                           int n_max, const pinfer_spec_params *sp, pinfer_spec_stats *stats) {
    int status;
    const int n = pinfer_generate_greedy_ex(c, prompt, n_prompt, out, n_max, sp, nullptr, stats, &status);
    return status != PINFER_OK ? status : n;
}

// ---- conversation state -------------------------------------------------------------------
// The reference's blob (engine/src/state.c:20-118), so blobs move between the two engines:
//   72-byte header: "PINFERS", version 2, n_past, kv_dtype, MTP rows, model dims, full-attention
//                   mask, pf_model_fingerprint of the file
//   per linear-attention layer (layer order): conv state [(K-1)][C], recurrent state [nv][dk][dv]
//   per full-attention layer: K rows [n_kv][n_past][hd], then V rows, at the storage precision
//                   (fp32, fp16, or int8 with each group's row scales after its rows)
//   MTP rows (mtp_rows of them): the MTP head's K and V rows, as the reference writes them
// Every generation ends with its deferred DeltaNet commit flushed, so the device state is
// complete whenever the API returns.
namespace {
struct StateHdr {
    char magic[8];
    uint32_t version, n_past, kv_dtype, mtp_rows;
    uint32_t n_layers, hidden, n_kv, head_dim, lk_heads, lv_heads, lk_dim, lv_dim, conv_k;
    uint32_t full_mask;
    uint64_t model_fp;
};
static_assert(sizeof(StateHdr) == 72, "state header layout of engine/src/state.c:24-30");
constexpr uint32_t kStateVersion = 2;

// bytes of one K or V row in the blob: hd elements at the storage precision, plus the int8
// scale (state.c:40-44, forward_kv.c:66-77)
size_t kv_row_bytes(const pinfer_ctx *c) {
    return c->kv_dtype == PINFER_KV_F16 ? (size_t)c->hd * 2
                                        : c->kv_dtype == PINFER_KV_I8 ? (size_t)c->hd + 4 : (size_t)c->hd * 4;
}

// IEEE binary16 bits of a float that binary16 represents exactly (the device rounded it when it
// stored the row), and back: sign, exponent rebias, subnormals, infinities, NaN (quiet, the top
// payload bits kept, as the reference's conversion writes them).
uint16_t f16_bits_exact(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u, e = (u >> 23) & 0xffu, man = u & 0x7fffffu;
    if (e == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0u));
    if (e == 0 && man == 0) return (uint16_t)sign;
    const int ex = (int)e - 127;
    if (ex >= -14) return (uint16_t)(sign | ((uint32_t)(ex + 15) << 10) | (man >> 13));
    // binary16 subnormal: value = m * 2^-24 with m < 1024
    const uint32_t full = man | 0x800000u;   // 1.man * 2^ex = full * 2^(ex - 23)
    return (uint16_t)(sign | (full >> (uint32_t)(-1 - ex)));
}
float f16_value(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    float v;
    if (e == 0x1fu) {
        const uint32_t u = sign | 0x7f800000u | (man << 13);
        memcpy(&v, &u, 4);
        return v;
    }
    v = e == 0 ? std::ldexp((float)man, -24) : std::ldexp((float)(man | 0x400u), (int)e - 25);
    return sign ? -v : v;
}

// the int8 code of a widened value v = q * s (q recovered exactly: |q| <= 127); a row whose
// scale is 0 (all zeros) or infinite (an infinity in the row: every value NaN) has codes 0
int8_t i8_code(float v, float s) {
    const float y = s != 0.0f ? std::rint(v / s) : 0.0f;
    return (int8_t)(y > 127.0f ? 127 : y < -127.0f ? -127 : y == y ? (int)y : 0);
}

size_t lin_state_floats(const pinfer_ctx *c) {
    return (size_t)std::max(c->K - 1, 1) * c->C + (size_t)c->nv * c->dk * c->dv;
}
size_t state_bytes(const pinfer_ctx *c, int n_past, int n_mtp = 0) {
    int n_full = 0;
    for (int l = 0; l < c->n_layers; l++) n_full += c->layers[l].is_full;
    return sizeof(StateHdr) + (size_t)c->n_lin * lin_state_floats(c) * 4 +
           (size_t)(n_full * (size_t)n_past + n_mtp) * 2 * c->nkv * kv_row_bytes(c);
}
int mtp_rows_saved(const pinfer_ctx *c) {   // state.c:51-53
    return c->mtp_ok && c->mtp_rows > 0 ? std::min(c->mtp_rows, c->n_past) : 0;
}
StateHdr state_header(const pinfer_ctx *c) {
    const PqHeader *h = &c->hdr;
    StateHdr s{};
    memcpy(s.magic, "PINFERS", 8);
    s.version = kStateVersion;
    s.n_past = (uint32_t)c->n_past;
    s.kv_dtype = (uint32_t)c->kv_dtype;
    s.mtp_rows = (uint32_t)mtp_rows_saved(c);
    s.n_layers = h->n_layers;
    s.hidden = h->hidden;
    s.n_kv = h->n_kv_heads;
    s.head_dim = h->head_dim;
    s.lk_heads = h->lin_k_heads;
    s.lv_heads = h->lin_v_heads;
    s.lk_dim = h->lin_k_dim;
    s.lv_dim = h->lin_v_dim;
    s.conv_k = h->conv_k;
    s.full_mask = h->full_attn_mask;
    s.model_fp = c->fp;
    return s;
}
// dir 0: device -> blob, 1: blob -> device; rows [0, n_past) of every cache
int state_copy(pinfer_ctx *c, char *cur, int n_past, int dir, int n_mtp = 0) {
    const auto kind = dir == 0 ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
    auto mv = [&](void *dev, size_t bytes) -> int {
        if (bytes == 0) return PINFER_OK;
        CUDA_OK(dir == 0 ? cudaMemcpyAsync(cur, dev, bytes, kind, c->stream)
                         : cudaMemcpyAsync(dev, cur, bytes, kind, c->stream));
        cur += bytes;
        return PINFER_OK;
    };
    int rc;
    const size_t conv = (size_t)std::max(c->K - 1, 1) * c->C * 4, rec = (size_t)c->nv * c->dk * c->dv * 4;
    for (int i = 0; i < c->n_lin; i++)
        if ((rc = mv(c->lin[i].conv_state, conv)) || (rc = mv(c->lin[i].rec, rec))) return rc;
    const size_t gstride = (size_t)c->max_ctx * c->hd;
    // n rows of group g of one cache: fp32 as they are; fp16 / int8 (the device holds the widened
    // values) converted to the stored form, int8 scales after the group's rows (state.c:64-83)
    std::vector<float> tmp;
    auto rows_of = [&](float *cache, float *scales, int g, int n) -> int {
        if (n <= 0) return PINFER_OK;
        float *dev = cache + g * gstride;
        const size_t cnt = (size_t)n * c->hd;
        if (c->kv_dtype == PINFER_KV_F32) return mv(dev, cnt * 4);
        tmp.resize(cnt);
        float *sc = scales ? scales + (size_t)g * c->max_ctx : nullptr;
        std::vector<float> s(c->kv_dtype == PINFER_KV_I8 ? (size_t)n : 0);
        if (dir == 0) {
            CUDA_OK(cudaMemcpyAsync(tmp.data(), dev, cnt * 4, cudaMemcpyDeviceToHost, c->stream));
            if (sc) CUDA_OK(cudaMemcpyAsync(s.data(), sc, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream));
            CUDA_OK(cudaStreamSynchronize(c->stream));
        }
        if (c->kv_dtype == PINFER_KV_F16) {
            uint16_t *h = reinterpret_cast<uint16_t *>(cur);
            for (size_t i = 0; i < cnt; i++) {
                if (dir == 0) {
                    const uint16_t b = f16_bits_exact(tmp[i]);
                    memcpy(h + i, &b, 2);
                } else {
                    uint16_t b;
                    memcpy(&b, h + i, 2);
                    tmp[i] = f16_value(b);
                }
            }
            cur += cnt * 2;
        } else {   // int8: q = value / scale (exact: |q| <= 127), NaN from a row with an infinity: 0
            int8_t *q = reinterpret_cast<int8_t *>(cur);
            float *bs = reinterpret_cast<float *>(cur + cnt);
            if (dir == 1) memcpy(s.data(), bs, (size_t)n * 4);
            for (int r = 0; r < n; r++)
                for (int i = 0; i < c->hd; i++) {
                    const size_t k = (size_t)r * c->hd + i;
                    if (dir == 0) {
                        q[k] = i8_code(tmp[k], s[r]);
                    } else {
                        tmp[k] = (float)q[k] * s[r];
                    }
                }
            if (dir == 0) memcpy(bs, s.data(), (size_t)n * 4);
            cur += cnt + (size_t)n * 4;
        }
        if (dir == 1) {
            CUDA_OK(cudaMemcpyAsync(dev, tmp.data(), cnt * 4, cudaMemcpyHostToDevice, c->stream));
            if (sc) CUDA_OK(cudaMemcpyAsync(sc, s.data(), (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
            CUDA_OK(cudaStreamSynchronize(c->stream));   // tmp and s are reused
        }
        return PINFER_OK;
    };
    for (int l = 0; l < c->n_layers; l++) {
        if (!c->layers[l].is_full) continue;
        for (int kv = 0; kv < 2; kv++)
            for (int g = 0; g < c->nkv; g++)
                if ((rc = rows_of(kv ? c->att[l].vc : c->att[l].kc, kv ? c->att[l].vs : c->att[l].ks, g, n_past)))
                    return rc;
    }
    for (int kv = 0; kv < 2 && n_mtp > 0; kv++)   // the MTP head's K then V rows
        for (int g = 0; g < c->nkv; g++)
            if ((rc = rows_of(kv ? c->mtp_att.vc : c->mtp_att.kc, kv ? c->mtp_att.vs : c->mtp_att.ks, g, n_mtp)))
                return rc;
    CUDA_OK(cudaStreamSynchronize(c->stream));
    return PINFER_OK;
}
}  // namespace

size_t pinfer_state_size(const pinfer_ctx *c) {
    return c ? state_bytes(c, c->n_past, mtp_rows_saved(c)) : 0;
}

int pinfer_state_save(const pinfer_ctx *c, void *buf, size_t cap) {
    if (!c || !buf) return PINFER_E_ARG;
    const int n_mtp = mtp_rows_saved(c);
    if (cap < state_bytes(c, c->n_past, n_mtp)) return PINFER_E_ARG;
    pinfer_ctx *m = const_cast<pinfer_ctx *>(c);   // the stream is used, the state is not changed
    const StateHdr h = state_header(c);
    memcpy(buf, &h, sizeof h);
    return state_copy(m, static_cast<char *>(buf) + sizeof h, c->n_past, 0, n_mtp);
}

int pinfer_state_load(pinfer_ctx *c, const void *buf, size_t len) {
    if (!c || !buf || len < sizeof(StateHdr)) return PINFER_E_ARG;
    StateHdr h;
    memcpy(&h, buf, sizeof h);
    const StateHdr mine = state_header(c);
    if (memcmp(h.magic, "PINFERS", 8) != 0 || h.version != kStateVersion) return PINFER_E_FORMAT;
    if (h.n_layers != mine.n_layers || h.hidden != mine.hidden || h.n_kv != mine.n_kv ||
        h.head_dim != mine.head_dim || h.lk_heads != mine.lk_heads || h.lv_heads != mine.lv_heads ||
        h.lk_dim != mine.lk_dim || h.lv_dim != mine.lv_dim || h.conv_k != mine.conv_k ||
        h.full_mask != mine.full_mask || h.kv_dtype != mine.kv_dtype || h.model_fp != mine.model_fp)
        return PINFER_E_FORMAT;   // another model file, or another KV storage format
    if (h.n_past > (uint32_t)c->max_ctx) return PINFER_E_CTX_FULL;
    if (h.mtp_rows > h.n_past || len < state_bytes(c, (int)h.n_past, (int)h.mtp_rows)) return PINFER_E_FORMAT;
    // MTP rows go to the MTP cache, or are dropped without the head (state.c:137-140)
    const int n_mtp = c->mtp_ok ? (int)h.mtp_rows : 0;
    launch_flush(c->lin, 0, c->lind, c->step, c->stream);   // drop any pending commit
    int rc = state_copy(c, const_cast<char *>(static_cast<const char *>(buf)) + sizeof h,
                        (int)h.n_past, 1, n_mtp);
    if (rc) return rc;
    // rows without saved values must not hold stale memory (state.c:149-152)
    if ((rc = zero_mtp_rows(c, n_mtp, (int)h.n_past)) || (rc = sync(c))) return rc;
    c->n_past = (int)h.n_past;
    c->mtp_rows = n_mtp;
    c->ck_valid = 0;   // the KV rows below the checkpoint were replaced
    return PINFER_OK;
}

int pinfer_checkpoint(pinfer_ctx *c) {
    if (!c) return PINFER_E_ARG;
    const size_t conv = (size_t)std::max(c->K - 1, 1) * c->C, rec = (size_t)c->nv * c->dk * c->dv;
    const size_t need = (size_t)c->n_lin * (conv + rec);
    if (!c->ck_buf) {
        if (cudaMalloc(&c->ck_buf, sizeof(float) * std::max<size_t>(need, 1)) != cudaSuccess) {
            c->ck_buf = nullptr;
            return PINFER_E_NOMEM;
        }
        c->ck_floats = need;
    }
    for (int i = 0; i < c->n_lin; i++) {
        CUDA_OK(cudaMemcpyAsync(c->ck_buf + i * (conv + rec), c->lin[i].conv_state, conv * 4, cudaMemcpyDeviceToDevice, c->stream));
        CUDA_OK(cudaMemcpyAsync(c->ck_buf + i * (conv + rec) + conv, c->lin[i].rec, rec * 4, cudaMemcpyDeviceToDevice, c->stream));
    }
    c->ck_valid = 1;
    c->ck_n_past = c->n_past;
    c->ck_mtp_rows = std::min(c->mtp_rows, c->n_past);
    return sync(c);
}

int pinfer_rewind(pinfer_ctx *c) {
    if (!c || !c->ck_valid) return PINFER_E_ARG;
    const size_t conv = (size_t)std::max(c->K - 1, 1) * c->C, rec = (size_t)c->nv * c->dk * c->dv;
    for (int i = 0; i < c->n_lin; i++) {
        CUDA_OK(cudaMemcpyAsync(c->lin[i].conv_state, c->ck_buf + i * (conv + rec), conv * 4, cudaMemcpyDeviceToDevice, c->stream));
        CUDA_OK(cudaMemcpyAsync(c->lin[i].rec, c->ck_buf + i * (conv + rec) + conv, rec * 4, cudaMemcpyDeviceToDevice, c->stream));
    }
    c->n_past = c->ck_n_past;
    c->mtp_rows = c->ck_mtp_rows;
    return sync(c);
}

void pinfer_checkpoint_clear(pinfer_ctx *c) {
    if (!c) return;
    cudaFree(c->ck_buf);
    c->ck_buf = nullptr;
    c->ck_valid = 0;
    c->ck_n_past = -1;
}

int pinfer_checkpoint_n_past(const pinfer_ctx *c) { return c && c->ck_valid ? c->ck_n_past : -1; }

int pinfer_n_vocab(const pinfer_ctx *c) { return c ? c->vocab : 0; }
int pinfer_n_past(const pinfer_ctx *c) { return c ? c->n_past : 0; }
int pinfer_eos_id(const pinfer_ctx *c) { return c ? c->eos : -1; }

// first maximum; NaN never chosen; a NaN in element 0 gives 0 (pf_argmax,
// engine/src/forward_ops.c:387-409)
int pinfer_argmax(const float *v, int n) {
    if (!v || n <= 0) return -1;
    float mx = v[0];
    for (int i = 0; i < n; i++)
        if (v[i] > mx) mx = v[i];
    for (int i = 0; i < n; i++)
        if (v[i] == mx) return i;
    return 0;
}

// ================================================================ B200 extensions (nb_b200.h)
const char *pinfer_b200_last_error(void) { return g_err.c_str(); }

int pinfer_b200_generate_synthetic_ex(pinfer_ctx *c, const int32_t *prompt, int n_prompt,
                                      int32_t *out, int n_max, int k, const int32_t *greedy,
                                      uint64_t seed, float p, int append,
                                      pinfer_spec_stats *stats, int *status, float *decode_ms) {
    int dummy;
    if (!status) status = &dummy;
    if (k < 0 || k > PINFER_SPEC_MAX_K || !(p >= 0.0f && p <= 1.0f) || (k > 0 && !greedy))
        return *status = PINFER_E_ARG;
    const unsigned p24 = (unsigned)std::min(16777216.0, std::floor((double)p * 16777216.0 + 0.5));
    GenRequest r{prompt, n_prompt, out, n_max, k, greedy, seed, p24, nullptr, append, {0, 0, 0}, 0.0f};
    const int n = generate_impl(c, &r, status);
    if (stats && n >= 0) {
        stats->rounds += r.stats[0];
        stats->drafted += r.stats[1];
        stats->accepted += r.stats[2];
    }
    if (decode_ms) *decode_ms = r.decode_ms;
    return n;
}

int pinfer_b200_generate_synthetic(pinfer_ctx *c, const int32_t *prompt, int n_prompt,
                                   int32_t *out, int n_max, int k, const int32_t *greedy,
                                   uint64_t seed, float p, pinfer_spec_stats *stats,
                                   int *status) {
    return pinfer_b200_generate_synthetic_ex(c, prompt, n_prompt, out, n_max, k, greedy, seed, p, 0,
                                             stats, status, nullptr);
}

int pinfer_b200_round_kernels(pinfer_ctx *c, int k) {
    if (!c || k < 0 || k > PINFER_SPEC_MAX_K) return PINFER_E_ARG;
    cudaGraphExec_t ex;
    if (round_graph(c, k, &ex)) return PINFER_E_NOMEM;
    // the graph is only instantiated; count its kernel nodes from a fresh capture
    cudaGraph_t g;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return PINFER_E_NOMEM;
    enqueue_forward(c, c->round_nmax[k], 2, false, true);
    launch_accept(c->step, c->d_greedy, c->d_out, c->stream);
    if (cudaStreamEndCapture(c->stream, &g) != cudaSuccess) return PINFER_E_NOMEM;
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    cudaGraphDestroy(g);
    return (int)n;
}

int pinfer_b200_forward_all(pinfer_ctx *c, const int32_t *tokens, int n, float *logits_all) {
    int rc = validate_tokens(c, tokens, n);
    if (rc) return rc;
    if (!logits_all) return PINFER_E_ARG;
    if (n > kMaxRows && c->shard_world == 1 && prefill_gemm_ok(c)) {   // chunks of up to 64 rows
        if ((rc = prefill_gemm(c, tokens, n, logits_all))) return rc;
        return sync(c);
    }
    for (int t0 = 0; t0 < n; t0 += kMaxRows) {
        const int nb = std::min(kMaxRows, n - t0);
        launch_set_pass(c->step, nb, c->n_past, 0, tokens + t0, c->stream);
        enqueue_forward(c, kMaxRows, 1);
        c->n_past += nb;
        CUDA_OK(cudaMemcpyAsync(logits_all + (size_t)t0 * c->vocab, c->logits, sizeof(float) * nb * (size_t)c->vocab,
                                cudaMemcpyDeviceToHost, c->stream));
    }
    return sync(c);
}

void *pinfer_b200_stream(pinfer_ctx *c) { return c ? (void *)c->stream : nullptr; }

int nb_test_kv_f16(int dir, const void *in, void *out, long long n) {
    if ((dir != 0 && dir != 1) || !in || !out || n < 0) return PINFER_E_ARG;
    for (long long i = 0; i < n; i++) {
        if (dir == 0) static_cast<uint16_t *>(out)[i] = f16_bits_exact(static_cast<const float *>(in)[i]);
        else static_cast<float *>(out)[i] = f16_value(static_cast<const uint16_t *>(in)[i]);
    }
    return PINFER_OK;
}

int nb_test_kv_i8(const float *v, const float *scales, int rows, int hd, int8_t *q) {
    if (!v || !scales || !q || rows < 0 || hd < 0) return PINFER_E_ARG;
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < hd; i++) q[(size_t)r * hd + i] = i8_code(v[(size_t)r * hd + i], scales[r]);
    return PINFER_OK;
}

pinfer_ctx *pinfer_b200_clone(const pinfer_ctx *src, int max_ctx, int *err) {
    int dummy;
    if (!err) err = &dummy;
    *err = PINFER_OK;
    if (!src || max_ctx < 0 || max_ctx > src->max_ctx) {
        set_err("pinfer_b200_clone: max_ctx must be in [0, the source's max_ctx]");
        *err = PINFER_E_ARG;
        return nullptr;
    }
    pinfer_ctx *c = new (std::nothrow) pinfer_ctx();
    if (!c) {
        *err = PINFER_E_NOMEM;
        return nullptr;
    }
    // the model: dimensions, parameter pointers (shared), no file
    c->H = src->H; c->ffn = src->ffn; c->n_layers = src->n_layers; c->vocab = src->vocab;
    c->nq = src->nq; c->nkv = src->nkv; c->hd = src->hd; c->rot = src->rot;
    c->nk = src->nk; c->nv = src->nv; c->dk = src->dk; c->dv = src->dv; c->K = src->K;
    c->kd = src->kd; c->vd = src->vd; c->C = src->C;
    c->max_ctx = max_ctx > 0 ? max_ctx : src->max_ctx;
    c->eps = src->eps; c->eos = src->eos; c->has_mtp = src->has_mtp; c->fp = src->fp; c->hdr = src->hdr;
    c->embed = src->embed; c->head = src->head; c->norm = src->norm;
    for (int l = 0; l < kMaxLayers; l++) {
        c->layers[l] = src->layers[l];
        c->lin[l] = src->lin[l];   // parameter pointers; the state buffers are replaced below
        c->att[l] = src->att[l];
    }
    c->n_lin = src->n_lin;
    c->mtp_ok = src->mtp_ok;   // the MTP head's parameters (its KV cache is allocated below)
    c->mtp_fc = src->mtp_fc;
    c->mtp_norm_emb = src->mtp_norm_emb;
    c->mtp_norm_hid = src->mtp_norm_hid;
    c->mtp_norm_out = src->mtp_norm_out;
    c->mtp_layer = src->mtp_layer;
    c->mtp_att.q_norm = src->mtp_att.q_norm;
    c->mtp_att.k_norm = src->mtp_att.k_norm;
    c->lind = src->lind;
    c->kv_dtype = src->kv_dtype;
    c->attd = src->attd;
    c->attd.max_ctx = c->max_ctx;   // the RoPE tables cover the source's (larger) context
    c->weights = src->weights;
    c->device = src->device;
    int rc = cudaSetDevice(c->device) == cudaSuccess ? PINFER_OK : PINFER_E_NOMEM;
    if (rc == PINFER_OK && cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_err("cannot create a CUDA stream");
        rc = PINFER_E_NOMEM;
    }
    if (rc == PINFER_OK) rc = alloc_state(c);
    if (rc == PINFER_OK && cudaStreamSynchronize(c->stream) != cudaSuccess) rc = PINFER_E_NOMEM;
    if (rc != PINFER_OK) {
        pinfer_free(c);
        *err = rc;
        return nullptr;
    }
    return c;
}

int pinfer_b200_nccl_id(void *id) {
    if (!id) return PINFER_E_ARG;
    char err[200];
    const NcclApi *n = nccl_api(err, sizeof err);
    if (!n) {
        set_err(err);
        return PINFER_E_NOMEM;
    }
    ncclUniqueId u;
    const ncclResult_t r = n->get_unique_id(&u);
    if (r != ncclSuccess) {
        set_err(n->error_string(r));
        return PINFER_E_NOMEM;
    }
    memcpy(id, &u, sizeof u);
    return PINFER_OK;
}

int pinfer_b200_shard_head(pinfer_ctx *c, int rank, int world, const void *id) {
    if (!c || world < 1 || rank < 0 || rank >= world || (world > 1 && !id)) return PINFER_E_ARG;
    if (world > 1 && c->vocab % (kPanelRows * world) != 0) {
        set_err("the vocabulary must split into equal shards of whole 32-row panels");
        return PINFER_E_ARG;
    }
    CUDA_OK(cudaStreamSynchronize(c->stream));
    drop_graphs(c);   // captured rounds hold the old head
    if (c->nccl) {
        const NcclApi *n = nccl_api(nullptr, 0);
        if (n) n->comm_destroy(c->nccl);
        c->nccl = nullptr;
    }
    c->shard_rank = 0;
    c->shard_world = 1;
    c->head_row0 = 0;
    if (world == 1) return PINFER_OK;
    char err[200];
    const NcclApi *n = nccl_api(err, sizeof err);
    if (!n) {
        set_err(err);
        return PINFER_E_NOMEM;
    }
    int rc;
    if (!c->d_keys && (rc = c->dalloc(&c->d_keys, sizeof(unsigned long long) * 2 * kMaxRows))) return rc;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    CUDA_OK(cudaSetDevice(c->device));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = n->comm_init_rank(&comm, world, u, rank);
    if (r != ncclSuccess) {
        set_err(n->error_string(r));
        return PINFER_E_NOMEM;
    }
    const int rows = c->vocab / world;
    c->nccl = comm;
    c->shard_rank = rank;
    c->shard_world = world;
    c->head_row0 = rank * rows;
    c->head_view = c->head;
    c->head_view.w = c->head.w + (size_t)(c->head_row0 / kPanelRows) * c->head.nsb * kUnitBytes;
    c->head_view.rows = rows;
    c->head_view.npanels = rows / kPanelRows;
    return PINFER_OK;
}

}  // extern "C"
