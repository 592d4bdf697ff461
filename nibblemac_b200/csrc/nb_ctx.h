// The context behind the opaque pinfer_ctx handle (host side): model dimensions, the weights
// on the device, per-context state and scratch. Shared by the engine sources; not public.
#pragma once
#include <cstdio>
#include <memory>
#include <mutex>
#include <vector>

#include "nb_engine.h"
#include "nb_model.h"
#include "nb_nccl.h"
#include "pinfer.h"

#define NB_CUDA_OK(call)                                                               \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            char b_[256];                                                              \
            snprintf(b_, sizeof b_, "CUDA error %s at %s:%d", cudaGetErrorString(e_),  \
                     __FILE__, __LINE__);                                              \
            nb::set_last_error(b_);                                                    \
            return PINFER_E_NOMEM;                                                     \
        }                                                                              \
    } while (0)

using nb::Mat;
using nb::PqFile;
using nb::PqHeader;
using nb::GemmW;
using nb::Act;
using nb::Step;
using nb::LinLayer;
using nb::LinDims;
using nb::AttnLayer;
using nb::AttnDims;
using nb::kMaxLayers;
using nb::kMaxRows;
using nb::GemmMaps;
using nb::SeqPass;

// ---------------------------------------------------------------- the context
// Device buffers of the model parameters (weights, norms, RoPE tables), shared by a context and
// its clones (pinfer_b200_clone) and freed with the last of them.
struct WeightStore {
    std::vector<void *> ptrs;
    // tensor-core tile images of the projections (nb_gemm.cu), made on the first prefill or
    // batch that needs them (ensure_gemm_tiles) and shared like the weights
    std::mutex tile_mu;
    bool tiles_ok = false, head_tile_ok = false;
    struct TileLayer {
        GemmW win, out, gu, down;   // gu: gate ++ up
    } tiles[kMaxLayers];
    GemmW head_tile;                // the whole LM head (logits of every prefill row)
    TileLayer mtp_tiles;            // the MTP head's decoder block (its gu: gate ++ up)
    GemmW mtp_fc_tile;              // the MTP head's input projection fc [e | h]
    ~WeightStore() {
        for (void *p : ptrs) cudaFree(p);
    }
};

// Rows of one prefill chunk through the tensor-core GEMMs (nb_prefill.cu), as the reference's
// batched prefill (engine/src/forward.c:154-165: chunks of ctx->batch <= 64 rows).
constexpr int kPrefillRows = 64;
constexpr int kPrefillSub = kPrefillRows / kMaxRows;   // 16-row sub-passes (Step blocks) per chunk

// A context's buffers for prefill chunks, allocated on first use.
struct PrefillScratch {
    bool ready = false;
    int ldy = 0;                              // y: W_in rows, or gate ++ up rows
    float *x = nullptr, *y = nullptr, *qbuf = nullptr;
    Act act_h, act_mid;
    GemmMaps maps_h, maps_ol, maps_oa, maps_f;
    Step *steps = nullptr;                    // [kPrefillSub]
    float *dn_recs = nullptr, *dn_o = nullptr;   // DeltaNet records and raw outputs of a chunk
    // MTP prompts: the chunk's final-normed rows, the MTP sub-passes (next tokens), [e | h] A8
    float *hn = nullptr;
    Step *msteps = nullptr;
    Act act_cat;
    GemmMaps maps_cat;
    SeqPass *d_pass = nullptr;                // [chunks of max_ctx][kPrefillSub]
    float *logits = nullptr;                  // [kPrefillRows][vocab] (forward_all), on first use
    unsigned long long *partial = nullptr;
    int *nan0 = nullptr;
};

struct pinfer_ctx {
    PqFile file;
    int H = 0, ffn = 0, n_layers = 0, vocab = 0, nq = 0, nkv = 0, hd = 0, rot = 0;
    int nk = 0, nv = 0, dk = 0, dv = 0, K = 0, kd = 0, vd = 0, C = 0;
    int max_ctx = 0, n_past = 0;
    int kv_dtype = 0;   // PINFER_KV_*: K / V rows rounded to this precision (held widened)
    float eps = 0;
    int eos = 0;
    int has_mtp = 0;
    uint64_t fp = 0;
    PqHeader hdr{};   // copy of the file header (the mapping is released after upload)
    cudaStream_t stream = nullptr;

    // weights (panel layout) and float parameters on the device
    Mat embed, head;
    struct Layer {
        int is_full = 0, lin = -1;
        Mat win, out, gate, up, down;   // win: qkv|z|b|a or q|k|v
        float *in_norm = nullptr, *post_norm = nullptr;
    } layers[kMaxLayers];
    float *norm = nullptr;
    LinLayer lin[kMaxLayers];
    AttnLayer att[kMaxLayers];
    int n_lin = 0;
    LinDims lind{};
    AttnDims attd{};
    std::vector<void *> allocs;                 // this context's buffers
    std::shared_ptr<WeightStore> weights;       // the model's parameters (shared with clones)

    // activations and scratch
    float *x = nullptr, *y = nullptr, *qbuf = nullptr, *logits = nullptr;
    Act act_h, act_mid;
    unsigned long long *partial = nullptr;
    int *nan0 = nullptr;
    unsigned long long *head_best = nullptr;   // [4][grid] per-CTA keys of the fused head argmax
    int *head_ctr = nullptr;                   // its grid counter (zero between launches)
    Step *step = nullptr;
    Step *h_step = nullptr;   // pinned mirror for reads
    int *d_out = nullptr, *d_greedy = nullptr;
    int out_cap = 0;

    // MTP draft head (speculative generation with k > 0): parameters shared with clones, KV
    // cache and buffers per context
    bool mtp_ok = false;
    Mat mtp_fc;
    float *mtp_norm_emb = nullptr, *mtp_norm_hid = nullptr, *mtp_norm_out = nullptr;
    Layer mtp_layer;
    AttnLayer mtp_att{};
    int mtp_rows = 0;                          // positions [0, mtp_rows) hold MTP KV rows
    float *hn = nullptr, *mrows = nullptr;     // [kMaxRows][H]: main final-normed rows, MTP output rows
    float *mcur = nullptr;                     // [H]: the m the next draft chain starts from
    Act act_cat;                               // [kMaxRows][2H]: MTP input rows, A8
    Step *msteps = nullptr;                    // [K+1]: 0 the pass over committed rows, s chain step s
    Mat mtp_head;                              // the head's first nv rows (draft vocabulary)
    cudaGraphExec_t round_graph_mtp[PINFER_SPEC_MAX_K + 1] = {};
    int graph_nv[PINFER_SPEC_MAX_K + 1] = {};
    int graph_ng[PINFER_SPEC_MAX_K + 1] = {};   // n-gram draft limit the MTP graph was sized for
    int graph_ad[PINFER_SPEC_MAX_K + 1] = {};   // the MTP graph holds the adaptive policy's kernels
    int graph_ng_ad[PINFER_SPEC_MAX_K + 1] = {};

    // graphs of one verify round per draft depth k (index k), no graph = not captured yet
    cudaGraphExec_t round_graph[PINFER_SPEC_MAX_K + 1] = {};
    cudaGraphExec_t round_graph_ng[PINFER_SPEC_MAX_K + 1] = {};   // n-gram drafts without MTP, by limit

    // prompt lookup: the device history's length and indexed prefix after the last generation
    int *ng_hist = nullptr, *ng_tab = nullptr;
    int ng_cap = 0, ng_bits = 0, ng_n = 0, ng_idx = 0;

    // vocab-sharded LM head (pinfer_b200_shard_head): this GPU's rows [head_row0, +head_view.rows)
    int device = 0;
    int shard_rank = 0, shard_world = 1, head_row0 = 0;
    Mat head_view;
    ncclComm_t nccl = nullptr;
    unsigned long long *d_keys = nullptr;   // [2][kMaxRows]: best key, row-0 NaN flag
    int round_nmax[PINFER_SPEC_MAX_K + 1] = {};

    PrefillScratch pf;

    // checkpoint slot (pinfer_checkpoint)
    float *ck_buf = nullptr;
    size_t ck_floats = 0;
    int ck_valid = 0, ck_n_past = -1, ck_mtp_rows = 0;

    template <class T>
    int dalloc(T **p, size_t bytes, bool weight = false) {
        void *q = nullptr;
        if (cudaMalloc(&q, bytes ? bytes : 16) != cudaSuccess) {
            nb::set_last_error("device allocation failed");
            return PINFER_E_NOMEM;
        }
        cudaMemset(q, 0, bytes ? bytes : 16);
        (weight ? weights->ptrs : allocs).push_back(q);
        *p = (T *)q;
        return PINFER_OK;
    }
};

// nb_prefill.cu
int ensure_gemm_tiles(pinfer_ctx *c, bool head);   // the shared tile images (head: the LM head's too)
bool prefill_gemm_ok(const pinfer_ctx *c);          // the model shape has the prefill kernels
// n rows (> kMaxRows worth it) at positions n_past.. in chunks of up to kPrefillRows rows;
// logits_all (host, [n][vocab], unsharded heads only) receives every row's logits; next (the
// tokens following rows 0..n-1) runs the MTP head's pass over each chunk too, filling its KV
// rows. Advances n_past; asynchronous on the context's stream unless logits are copied out.
int prefill_gemm(pinfer_ctx *c, const int32_t *tokens, int n, float *logits_all, const int32_t *next = nullptr);
