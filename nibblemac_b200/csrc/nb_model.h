// .pq file structures and the validated view of a loaded model (host side).
// On-disk layout: engine/FORMAT.md; structs engine/src/pq_format.h:32-62 (same field order).
#pragma once
#include <cstddef>
#include <cstdint>

namespace nb {

enum : uint32_t { kPqF32 = 0, kPqBF16 = 1, kPqQ4K = 4 };

struct PqHeader {
    char magic[8];
    uint32_t version;
    uint32_t n_tensors;
    uint64_t dir_offset;
    uint64_t data_offset;
    uint32_t arch;
    uint32_t hidden, n_layers, vocab, ffn;
    uint32_t n_heads, n_kv_heads, head_dim, rot_dim;
    uint32_t lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim, conv_k;
    uint32_t full_attn_mask;
    uint32_t eos_id;
    uint32_t tied_embeddings;
    uint32_t has_mtp;
    float rms_eps;
    float rope_theta;
};

struct PqEntry {
    char name[80];
    uint32_t dtype;
    uint32_t ndim;
    uint32_t shape[4];
    uint64_t offset;
    uint64_t nbytes;
    uint8_t reserved[8];
};
static_assert(sizeof(PqEntry) == 128, "pq_tensor_entry is 128 bytes");

struct PqMat {
    const uint8_t *data = nullptr;   // Q4K_G32 tiles in the mapped file
    int rows = 0, cols = 0;
};

struct PqLayer {
    int is_full = 0;
    const float *in_norm = nullptr, *post_norm = nullptr;
    PqMat gate, up, down;
    PqMat qkv, z, b, a, out;
    const float *conv_w = nullptr, *A_log = nullptr, *A = nullptr, *dt_bias = nullptr, *lin_norm = nullptr;
    PqMat q, k, v, o;
    const float *q_norm = nullptr, *k_norm = nullptr;
};

// The MTP draft head (engine/src/mtp.c:8-32): fc [H][2H], three norms, one full-attention block.
struct PqMtp {
    bool ok = false;   // every mtp.* tensor present with the right shape
    PqMat fc;
    const float *norm_emb = nullptr, *norm_hid = nullptr, *norm_out = nullptr;
    PqLayer layer;
};

struct PqFile {
    void *map = nullptr;
    size_t map_bytes = 0;
    const PqHeader *hdr = nullptr;
    const PqEntry *dir = nullptr;
    PqMat embed, head;
    const float *norm = nullptr;
    PqLayer layers[32];
    PqMtp mtp;

    int open_file(const char *path);   // PINFER_OK / PINFER_E_IO / PINFER_E_FORMAT
    void close_file();
    const PqEntry *find(const char *name) const;
    int vec(const char *name, uint32_t n, const float **out) const;
    int mat(const char *name, uint32_t rows, uint32_t cols, PqMat *out) const;
    uint64_t fingerprint() const;
};

}  // namespace nb
