// .pq loader for the B200 engine: map the file, validate header and directory exactly as the
// reference loader does (engine/src/model.c), then expose typed views for the upload.
//
// The checks follow check_header (model.c:116-139), check_directory (:60-84), entry_bytes
// (:31-55), pf_model_vec / pf_model_mat (:86-110) and build_layer (:156-205), with the same
// error codes: PINFER_E_IO when the file cannot be opened or mapped, PINFER_E_FORMAT for
// anything malformed. On top of the reference's engine limits this build runs Q4K_G32
// matrices only and Gated DeltaNet heads of 128 x 128.
#include "nb_model.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "pinfer.h"

namespace nb {

static int fail(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fputs("pinfer: ", stderr);
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
    return PINFER_E_FORMAT;
}

const PqEntry *PqFile::find(const char *name) const {
    for (uint32_t i = 0; i < hdr->n_tensors; i++)
        if (strcmp(dir[i].name, name) == 0) return &dir[i];
    return nullptr;
}

// entry_bytes (model.c:31-55): the size the dtype and shape imply, built against the file size
static int entry_bytes(const PqEntry *e, uint64_t limit, uint64_t *bytes) {
    const uint64_t es = e->dtype == kPqF32 ? 4 : e->dtype == kPqBF16 ? 2 : 0;
    if (es) {
        uint64_t n = es;
        for (uint32_t d = 0; d < e->ndim; d++) {
            if (!e->shape[d]) return fail("%s: zero dimension", e->name);
            if (n > limit / e->shape[d]) return fail("%s: shape larger than the file", e->name);
            n *= e->shape[d];
        }
        *bytes = n;
        return PINFER_OK;
    }
    uint64_t sb = 0;
    if (e->dtype == 2) sb = 1088;
    else if (e->dtype == 3 || e->dtype == 4) sb = 576;
    if (!sb) return fail("%s: unknown dtype %u", e->name, e->dtype);
    const uint64_t rows = e->shape[0], cols = e->shape[1];
    if (e->ndim != 2 || !rows || !cols || rows % 4 || cols % 256)
        return fail("%s: quantized dtype %u needs a [rows %% 4, cols %% 256] matrix", e->name, e->dtype);
    const uint64_t tiles = rows / 4 * (cols / 256);
    if (tiles > limit / sb) return fail("%s: shape larger than the file", e->name);
    *bytes = tiles * sb;
    return PINFER_OK;
}

static int check_header(const PqHeader *h) {   // model.c:116-139
    if (memcmp(h->magic, "PINFERQ", 8) != 0) return fail("bad magic");
    if (h->version != 1) return fail("unsupported version %u", h->version);
    if (h->arch != 1) return fail("unsupported arch %u", h->arch);
    if (!h->hidden || h->hidden > 65536u || !h->ffn || h->ffn > 65536u || !h->vocab ||
        h->vocab > (1u << 21) || !h->n_layers || h->n_layers > 32u)
        return fail("bad model dimensions");
    if (h->eos_id >= h->vocab) return fail("eos_id %u outside the vocabulary", h->eos_id);
    if (!h->n_heads || h->n_heads > 256u || !h->n_kv_heads || h->n_heads % h->n_kv_heads ||
        !h->head_dim || h->head_dim > 1024u || h->rot_dim % 2 || h->rot_dim > h->head_dim)
        return fail("bad attention dimensions");
    if (!h->lin_k_heads || h->lin_k_heads > 256u || !h->lin_v_heads || h->lin_v_heads > 256u ||
        h->lin_v_heads % h->lin_k_heads || !h->lin_k_dim || h->lin_k_dim > 1024u ||
        !h->lin_v_dim || h->lin_v_dim > 1024u || h->conv_k < 1 || h->conv_k > 8u)
        return fail("bad linear-attention dimensions");
    if (h->tied_embeddings > 1) return fail("bad tied_embeddings %u", h->tied_embeddings);
    if (!(h->rms_eps > 0.0f) || !std::isfinite(h->rms_eps) || !(h->rope_theta > 0.0f) ||
        !std::isfinite(h->rope_theta))
        return fail("bad eps / rope_theta");
    return PINFER_OK;
}

static int check_directory(PqFile *m) {   // model.c:60-84
    const PqHeader *h = m->hdr;
    const uint64_t size = m->map_bytes;
    if (h->dir_offset < sizeof(PqHeader) || h->dir_offset > size || h->dir_offset % 8 ||
        (uint64_t)h->n_tensors * sizeof(PqEntry) > size - h->dir_offset)
        return fail("tensor directory out of bounds or misaligned");
    if (h->data_offset > size) return fail("data_offset out of bounds");
    m->dir = (const PqEntry *)((const char *)m->map + h->dir_offset);
    for (uint32_t i = 0; i < h->n_tensors; i++) {
        const PqEntry *e = &m->dir[i];
        if (!memchr(e->name, 0, sizeof e->name)) return fail("tensor %u: name not terminated", i);
        if (e->ndim < 1 || e->ndim > 4) return fail("%s: bad ndim %u", e->name, e->ndim);
        if (e->offset % 64 || e->offset < h->data_offset || e->offset > size ||
            e->nbytes > size - e->offset)
            return fail("%s: data out of bounds or misaligned", e->name);
        uint64_t want = 0;
        if (entry_bytes(e, size, &want) != PINFER_OK) return PINFER_E_FORMAT;
        if (want != e->nbytes)
            return fail("%s: nbytes %llu != %llu for dtype %u and its shape", e->name,
                        (unsigned long long)e->nbytes, (unsigned long long)want, e->dtype);
    }
    return PINFER_OK;
}

int PqFile::vec(const char *name, uint32_t n, const float **out) const {
    const PqEntry *e = find(name);
    if (!e) return fail("missing tensor %s", name);
    if (e->dtype != kPqF32 || e->ndim != 1 || e->shape[0] != n) return fail("%s: expected F32 [%u]", name, n);
    *out = (const float *)((const char *)map + e->offset);
    return PINFER_OK;
}

int PqFile::mat(const char *name, uint32_t rows, uint32_t cols, PqMat *out) const {
    const PqEntry *e = find(name);
    if (!e) return fail("missing tensor %s", name);
    if (e->ndim != 2 || e->shape[0] != rows || e->shape[1] != cols)
        return fail("%s: expected shape [%u, %u]", name, rows, cols);
    if (e->dtype != kPqQ4K)
        return fail("%s: dtype %u not supported by this build (Q4K_G32 matrices only)", name, e->dtype);
    out->data = (const uint8_t *)map + e->offset;
    out->rows = (int)rows;
    out->cols = (int)cols;
    return PINFER_OK;
}

// model.c:156-205; prefix "layers.<i>." for the main layers, "mtp.layers.0." (always a
// full-attention block) for the MTP head's.
static int build_layer(const PqFile &m, int i, PqLayer *L, const char *prefix = nullptr) {
    const PqHeader *h = m.hdr;
    char nm[160];
    int rc = 0;
    auto N = [&](const char *s) {
        if (prefix) snprintf(nm, sizeof nm, "%s%s", prefix, s);
        else snprintf(nm, sizeof nm, "layers.%d.%s", i, s);
        return nm;
    };
    const uint32_t H = h->hidden;
    L->is_full = prefix ? 1 : (h->full_attn_mask >> i) & 1;
    rc |= m.vec(N("input_layernorm.weight"), H, &L->in_norm);
    rc |= m.vec(N("post_attention_layernorm.weight"), H, &L->post_norm);
    rc |= m.mat(N("mlp.gate_proj.weight"), h->ffn, H, &L->gate);
    rc |= m.mat(N("mlp.up_proj.weight"), h->ffn, H, &L->up);
    rc |= m.mat(N("mlp.down_proj.weight"), H, h->ffn, &L->down);
    if (L->is_full) {
        const uint32_t hd = h->head_dim;
        rc |= m.mat(N("self_attn.q_proj.weight"), h->n_heads * hd * 2, H, &L->q);
        rc |= m.mat(N("self_attn.k_proj.weight"), h->n_kv_heads * hd, H, &L->k);
        rc |= m.mat(N("self_attn.v_proj.weight"), h->n_kv_heads * hd, H, &L->v);
        rc |= m.mat(N("self_attn.o_proj.weight"), H, h->n_heads * hd, &L->o);
        rc |= m.vec(N("self_attn.q_norm.weight"), hd, &L->q_norm);
        rc |= m.vec(N("self_attn.k_norm.weight"), hd, &L->k_norm);
    } else {
        const uint32_t kd = h->lin_k_heads * h->lin_k_dim, vd = h->lin_v_heads * h->lin_v_dim;
        const uint32_t conv_dim = 2 * kd + vd;
        rc |= m.mat(N("linear_attn.in_proj_qkv.weight"), conv_dim, H, &L->qkv);
        rc |= m.mat(N("linear_attn.in_proj_z.weight"), vd, H, &L->z);
        rc |= m.mat(N("linear_attn.in_proj_b.weight"), h->lin_v_heads, H, &L->b);
        rc |= m.mat(N("linear_attn.in_proj_a.weight"), h->lin_v_heads, H, &L->a);
        rc |= m.mat(N("linear_attn.out_proj.weight"), H, vd, &L->out);
        const bool has_a = m.find(N("linear_attn.A")) != nullptr;
        if (has_a && m.find(N("linear_attn.A_log"))) return fail("layer %d: both linear_attn.A and linear_attn.A_log", i);
        if (has_a) rc |= m.vec(N("linear_attn.A"), h->lin_v_heads, &L->A);
        else rc |= m.vec(N("linear_attn.A_log"), h->lin_v_heads, &L->A_log);
        rc |= m.vec(N("linear_attn.dt_bias"), h->lin_v_heads, &L->dt_bias);
        rc |= m.vec(N("linear_attn.norm.weight"), h->lin_v_dim, &L->lin_norm);
        const PqEntry *e = m.find(N("linear_attn.conv1d.weight"));
        if (!e || e->dtype != kPqF32 || e->ndim != 2 || e->shape[0] != conv_dim || e->shape[1] != h->conv_k)
            return fail("layer %d: bad or missing conv1d.weight", i);
        L->conv_w = (const float *)((const char *)m.map + e->offset);
    }
    return rc ? PINFER_E_FORMAT : PINFER_OK;
}

int PqFile::open_file(const char *path) {
    close_file();
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        perror(path);
        return PINFER_E_IO;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 4096) {
        ::close(fd);
        fprintf(stderr, "pinfer: %s: too small for a .pq file\n", path);
        return PINFER_E_FORMAT;
    }
    void *p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) {
        perror("mmap");
        return PINFER_E_IO;
    }
    map = p;
    map_bytes = (size_t)st.st_size;
    hdr = (const PqHeader *)p;
    int rc = check_header(hdr);
    if (rc == PINFER_OK) rc = check_directory(this);
    if (rc == PINFER_OK) rc = mat("embed_tokens.weight", hdr->vocab, hdr->hidden, &embed);
    if (rc == PINFER_OK) {
        head = embed;
        if (!hdr->tied_embeddings) rc = mat("lm_head.weight", hdr->vocab, hdr->hidden, &head);
    }
    if (rc == PINFER_OK) rc = vec("norm.weight", hdr->hidden, &norm);
    for (uint32_t i = 0; rc == PINFER_OK && i < hdr->n_layers; i++) rc = build_layer(*this, (int)i, &layers[i]);
    if (rc != PINFER_OK) {
        close_file();
        return rc;
    }
    // The MTP head is mapped lazily by the reference (pf_mtp_init at the first speculative
    // generation), so a missing or malformed head does not fail the load: generation with
    // k > 0 then returns PINFER_E_FORMAT.
    if (hdr->has_mtp) {
        const uint32_t H = hdr->hidden;
        int m = PINFER_OK;
        m |= find("mtp.fc.weight") ? mat("mtp.fc.weight", H, 2 * H, &mtp.fc) : PINFER_E_FORMAT;
        m |= find("mtp.pre_fc_norm_embedding.weight") ? vec("mtp.pre_fc_norm_embedding.weight", H, &mtp.norm_emb) : PINFER_E_FORMAT;
        m |= find("mtp.pre_fc_norm_hidden.weight") ? vec("mtp.pre_fc_norm_hidden.weight", H, &mtp.norm_hid) : PINFER_E_FORMAT;
        m |= find("mtp.norm.weight") ? vec("mtp.norm.weight", H, &mtp.norm_out) : PINFER_E_FORMAT;
        if (m == PINFER_OK && find("mtp.layers.0.self_attn.q_proj.weight"))
            m = build_layer(*this, 0, &mtp.layer, "mtp.layers.0.");
        else
            m = PINFER_E_FORMAT;
        mtp.ok = m == PINFER_OK;
    }
    return rc;
}

void PqFile::close_file() {
    if (map) munmap(map, map_bytes);
    map = nullptr;
    map_bytes = 0;
    hdr = nullptr;
    dir = nullptr;
    for (auto &L : layers) L = PqLayer();
    mtp = PqMtp();
}

// pf_model_fingerprint (model.c:142-154): FNV-1a over the header, the directory and three
// 64-byte samples of every tensor.
uint64_t PqFile::fingerprint() const {
    auto fnv = [](uint64_t h, const void *p, size_t n) {
        const unsigned char *b = (const unsigned char *)p;
        for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 1099511628211ull;
        return h;
    };
    uint64_t h = fnv(14695981039346656037ull, hdr, sizeof(PqHeader));
    h = fnv(h, dir, (size_t)hdr->n_tensors * sizeof(PqEntry));
    for (uint32_t i = 0; i < hdr->n_tensors; i++) {
        const PqEntry *e = &dir[i];
        const unsigned char *d = (const unsigned char *)map + e->offset;
        const size_t n = (size_t)e->nbytes, s = n < 64 ? n : 64;
        h = fnv(h, d, s);
        h = fnv(h, d + (n - s) / 2, s);
        h = fnv(h, d + (n - s), s);
    }
    return h;
}

}  // namespace nb
