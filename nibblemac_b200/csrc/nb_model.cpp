// .pq reader for the B200 engine: map the file, validate it, and bind typed views of the
// tensors the engine uploads.
//
// The acceptance rules are the reference loader's (engine/src/model.c: header limits :116-139,
// directory bounds :60-84, the size a dtype and shape imply :31-55, per-layer tensor names and
// shapes :156-205): a file the reference refuses is refused here with the same code
// (PINFER_E_IO when it cannot be opened or mapped, PINFER_E_FORMAT for anything malformed), so
// callers see the same outcome from either engine. The rules are written as tables: header
// fields with their ranges, dtypes with their storage sizes, and per-layer tensor lists, checked
// by a few generic routines. On top of the reference's limits this build runs Q4K_G32 matrices
// only (and Gated DeltaNet heads of 128 x 128, checked at upload).
#include "nb_model.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>

#include "pinfer.h"

namespace nb {
namespace {

// Malformed input: one diagnostic line on stderr, PINFER_E_FORMAT.
int reject(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "pinfer (.pq): ");
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
    return PINFER_E_FORMAT;
}

// ---- header ------------------------------------------------------------------------------
// Dimension fields and their accepted ranges. Fields related to one another (divisibility,
// eos inside the vocabulary, rotary part inside the head) are checked after the table.
struct FieldRange {
    const char *field;
    uint32_t PqHeader::*member;
    uint32_t lo, hi;
};
const FieldRange kHeaderRanges[] = {
    {"hidden", &PqHeader::hidden, 1, 65536},
    {"ffn", &PqHeader::ffn, 1, 65536},
    {"vocab", &PqHeader::vocab, 1, 1u << 21},
    {"n_layers", &PqHeader::n_layers, 1, 32},
    {"n_heads", &PqHeader::n_heads, 1, 256},
    {"n_kv_heads", &PqHeader::n_kv_heads, 1, 0xffffffffu},
    {"head_dim", &PqHeader::head_dim, 1, 1024},
    {"rot_dim", &PqHeader::rot_dim, 0, 0xffffffffu},
    {"lin_k_heads", &PqHeader::lin_k_heads, 1, 256},
    {"lin_v_heads", &PqHeader::lin_v_heads, 1, 256},
    {"lin_k_dim", &PqHeader::lin_k_dim, 1, 1024},
    {"lin_v_dim", &PqHeader::lin_v_dim, 1, 1024},
    {"conv_k", &PqHeader::conv_k, 1, 8},
    {"tied_embeddings", &PqHeader::tied_embeddings, 0, 1},
};

int validate_header(const PqHeader &h) {
    if (memcmp(h.magic, "PINFERQ", 8) != 0) return reject("not a .pq file (magic)");
    if (h.version != 1) return reject("format version %u (this reader knows 1)", h.version);
    if (h.arch != 1) return reject("architecture id %u (this reader knows 1)", h.arch);
    for (const FieldRange &f : kHeaderRanges) {
        const uint32_t v = h.*f.member;
        if (v < f.lo || v > f.hi) return reject("header field %s = %u outside [%u, %u]", f.field, v, f.lo, f.hi);
    }
    struct Relation {
        bool ok;
        const char *what;
    };
    const Relation rel[] = {
        {h.eos_id < h.vocab, "eos_id must be a vocabulary id"},
        {h.n_heads % h.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads"},
        {h.rot_dim % 2 == 0 && h.rot_dim <= h.head_dim, "rot_dim must be even and at most head_dim"},
        {h.lin_v_heads % h.lin_k_heads == 0, "lin_v_heads must be a multiple of lin_k_heads"},
        {h.rms_eps > 0.0f && std::isfinite(h.rms_eps), "rms_eps must be positive and finite"},
        {h.rope_theta > 0.0f && std::isfinite(h.rope_theta), "rope_theta must be positive and finite"},
    };
    for (const Relation &r : rel)
        if (!r.ok) return reject("header: %s", r.what);
    return PINFER_OK;
}

// ---- directory ---------------------------------------------------------------------------
// Storage of each dtype: dense types by element, quantised types by 4-row x 256-column tile.
struct DtypeSize {
    uint32_t id;
    uint32_t elem;   // bytes per element (dense), or 0
    uint32_t tile;   // bytes per 4 x 256 tile (quantised), or 0
};
const DtypeSize kDtypes[] = {{kPqF32, 4, 0}, {kPqBF16, 2, 0}, {2, 0, 1088}, {3, 0, 576}, {kPqQ4K, 0, 576}};

// a * b when it stays at or below `limit` (no wrap); false otherwise
bool mul_capped(uint64_t a, uint64_t b, uint64_t limit, uint64_t *out) {
    if (b != 0 && a > limit / b) return false;
    *out = a * b;
    return true;
}

// The byte count an entry's dtype and shape imply, bounded by the file size.
int implied_bytes(const PqEntry &e, uint64_t file_bytes, uint64_t *bytes) {
    const DtypeSize *t = nullptr;
    for (const DtypeSize &d : kDtypes)
        if (d.id == e.dtype) t = &d;
    if (!t) return reject("%s: dtype %u is not a .pq dtype", e.name, e.dtype);
    if (t->elem) {
        uint64_t n = t->elem;
        for (uint32_t i = 0; i < e.ndim; i++) {
            if (e.shape[i] == 0) return reject("%s: dimension %u is empty", e.name, i);
            if (!mul_capped(n, e.shape[i], file_bytes, &n)) return reject("%s: shape exceeds the file", e.name);
        }
        *bytes = n;
        return PINFER_OK;
    }
    const uint64_t rows = e.shape[0], cols = e.shape[1];
    if (e.ndim != 2 || rows == 0 || cols == 0 || rows % 4 != 0 || cols % 256 != 0)
        return reject("%s: a quantised tensor is a matrix of rows %% 4 == 0, cols %% 256 == 0", e.name);
    if (!mul_capped(rows / 4 * (cols / 256), t->tile, file_bytes, bytes))
        return reject("%s: shape exceeds the file", e.name);
    return PINFER_OK;
}

int validate_directory(PqFile &f) {
    const PqHeader &h = *f.hdr;
    const uint64_t size = f.map_bytes;
    const bool dir_fits = h.dir_offset >= sizeof(PqHeader) && h.dir_offset <= size && h.dir_offset % 8 == 0 &&
                          (uint64_t)h.n_tensors * sizeof(PqEntry) <= size - h.dir_offset;
    if (!dir_fits) return reject("directory (offset %llu, %u entries) does not fit the file",
                                 (unsigned long long)h.dir_offset, h.n_tensors);
    if (h.data_offset > size) return reject("data offset %llu past the end of the file", (unsigned long long)h.data_offset);
    f.dir = reinterpret_cast<const PqEntry *>(static_cast<const char *>(f.map) + h.dir_offset);
    for (uint32_t i = 0; i < h.n_tensors; i++) {
        const PqEntry &e = f.dir[i];
        if (!memchr(e.name, 0, sizeof e.name)) return reject("directory entry %u: name has no terminator", i);
        if (e.ndim < 1 || e.ndim > 4) return reject("%s: %u dimensions (1 to 4 allowed)", e.name, e.ndim);
        const bool placed = e.offset % 64 == 0 && e.offset >= h.data_offset && e.offset <= size &&
                            e.nbytes <= size - e.offset;
        if (!placed) return reject("%s: data range not 64-byte aligned inside the data section", e.name);
        uint64_t want = 0;
        if (implied_bytes(e, size, &want) != PINFER_OK) return PINFER_E_FORMAT;
        if (want != e.nbytes)
            return reject("%s: stores %llu bytes, its dtype and shape need %llu", e.name,
                          (unsigned long long)e.nbytes, (unsigned long long)want);
    }
    return PINFER_OK;
}

// ---- per-layer tensors ---------------------------------------------------------------------
using DimOf = uint32_t (*)(const PqHeader &);
struct MatSpec {
    const char *suffix;
    DimOf rows, cols;
    PqMat PqLayer::*dst;
};
struct VecSpec {
    const char *suffix;
    DimOf len;
    const float *PqLayer::*dst;
};

uint32_t dim_hidden(const PqHeader &h) { return h.hidden; }
uint32_t dim_ffn(const PqHeader &h) { return h.ffn; }
uint32_t dim_q2(const PqHeader &h) { return h.n_heads * h.head_dim * 2; }   // query | gate per head
uint32_t dim_q(const PqHeader &h) { return h.n_heads * h.head_dim; }
uint32_t dim_kv(const PqHeader &h) { return h.n_kv_heads * h.head_dim; }
uint32_t dim_head(const PqHeader &h) { return h.head_dim; }
uint32_t dim_conv(const PqHeader &h) { return 2 * h.lin_k_heads * h.lin_k_dim + h.lin_v_heads * h.lin_v_dim; }
uint32_t dim_vd(const PqHeader &h) { return h.lin_v_heads * h.lin_v_dim; }
uint32_t dim_vheads(const PqHeader &h) { return h.lin_v_heads; }
uint32_t dim_vdim(const PqHeader &h) { return h.lin_v_dim; }

const VecSpec kBlockVecs[] = {{"input_layernorm.weight", dim_hidden, &PqLayer::in_norm},
                              {"post_attention_layernorm.weight", dim_hidden, &PqLayer::post_norm}};
const MatSpec kMlpMats[] = {{"mlp.gate_proj.weight", dim_ffn, dim_hidden, &PqLayer::gate},
                            {"mlp.up_proj.weight", dim_ffn, dim_hidden, &PqLayer::up},
                            {"mlp.down_proj.weight", dim_hidden, dim_ffn, &PqLayer::down}};
const MatSpec kAttnMats[] = {{"self_attn.q_proj.weight", dim_q2, dim_hidden, &PqLayer::q},
                             {"self_attn.k_proj.weight", dim_kv, dim_hidden, &PqLayer::k},
                             {"self_attn.v_proj.weight", dim_kv, dim_hidden, &PqLayer::v},
                             {"self_attn.o_proj.weight", dim_hidden, dim_q, &PqLayer::o}};
const VecSpec kAttnVecs[] = {{"self_attn.q_norm.weight", dim_head, &PqLayer::q_norm},
                             {"self_attn.k_norm.weight", dim_head, &PqLayer::k_norm}};
const MatSpec kLinMats[] = {{"linear_attn.in_proj_qkv.weight", dim_conv, dim_hidden, &PqLayer::qkv},
                            {"linear_attn.in_proj_z.weight", dim_vd, dim_hidden, &PqLayer::z},
                            {"linear_attn.in_proj_b.weight", dim_vheads, dim_hidden, &PqLayer::b},
                            {"linear_attn.in_proj_a.weight", dim_vheads, dim_hidden, &PqLayer::a},
                            {"linear_attn.out_proj.weight", dim_hidden, dim_vd, &PqLayer::out}};
const VecSpec kLinVecs[] = {{"linear_attn.dt_bias", dim_vheads, &PqLayer::dt_bias},
                            {"linear_attn.norm.weight", dim_vdim, &PqLayer::lin_norm}};

// Binds one decoder block whose tensor names start with `prefix`. Every tensor is checked (the
// first failure does not stop the others, so each is reported), then the block fails or passes.
int bind_block(const PqFile &f, const char *prefix, bool full, PqLayer *L) {
    const PqHeader &h = *f.hdr;
    char name[160];
    auto named = [&](const char *suffix) {
        snprintf(name, sizeof name, "%s%s", prefix, suffix);
        return name;
    };
    int bad = 0;
    auto mats = [&](const MatSpec *s, size_t n) {
        for (size_t i = 0; i < n; i++) bad |= f.mat(named(s[i].suffix), s[i].rows(h), s[i].cols(h), &(L->*s[i].dst));
    };
    auto vecs = [&](const VecSpec *s, size_t n) {
        for (size_t i = 0; i < n; i++) bad |= f.vec(named(s[i].suffix), s[i].len(h), &(L->*s[i].dst));
    };
    L->is_full = full;
    vecs(kBlockVecs, 2);
    mats(kMlpMats, 3);
    if (full) {
        mats(kAttnMats, 4);
        vecs(kAttnVecs, 2);
        return bad ? PINFER_E_FORMAT : PINFER_OK;
    }
    mats(kLinMats, 5);
    vecs(kLinVecs, 2);
    // the decay parameter comes either as A itself or as A_log (A = -exp(A_log)), never both
    const bool has_a = f.find(named("linear_attn.A")) != nullptr;
    const bool has_alog = f.find(named("linear_attn.A_log")) != nullptr;
    if (has_a && has_alog) return reject("%s: carries both linear_attn.A and linear_attn.A_log", prefix);
    bad |= has_a ? f.vec(named("linear_attn.A"), h.lin_v_heads, &L->A)
                 : f.vec(named("linear_attn.A_log"), h.lin_v_heads, &L->A_log);
    const PqEntry *conv = f.find(named("linear_attn.conv1d.weight"));
    if (!conv || conv->dtype != kPqF32 || conv->ndim != 2 || conv->shape[0] != dim_conv(h) || conv->shape[1] != h.conv_k)
        return reject("%slinear_attn.conv1d.weight: needs F32 [%u, %u]", prefix, dim_conv(h), h.conv_k);
    L->conv_w = reinterpret_cast<const float *>(static_cast<const char *>(f.map) + conv->offset);
    return bad ? PINFER_E_FORMAT : PINFER_OK;
}

}  // namespace

const PqEntry *PqFile::find(const char *name) const {
    for (uint32_t i = 0; i < hdr->n_tensors; i++)
        if (strcmp(dir[i].name, name) == 0) return &dir[i];
    return nullptr;
}

int PqFile::vec(const char *name, uint32_t n, const float **out) const {
    const PqEntry *e = find(name);
    if (!e) return reject("tensor %s is missing", name);
    if (e->dtype != kPqF32 || e->ndim != 1 || e->shape[0] != n) return reject("%s: needs F32 [%u]", name, n);
    *out = reinterpret_cast<const float *>(static_cast<const char *>(map) + e->offset);
    return PINFER_OK;
}

int PqFile::mat(const char *name, uint32_t rows, uint32_t cols, PqMat *out) const {
    const PqEntry *e = find(name);
    if (!e) return reject("tensor %s is missing", name);
    if (e->ndim != 2 || e->shape[0] != rows || e->shape[1] != cols)
        return reject("%s: needs a [%u, %u] matrix", name, rows, cols);
    if (e->dtype != kPqQ4K)
        return reject("%s: dtype %u; the B200 engine reads Q4K_G32 matrices only", name, e->dtype);
    out->data = static_cast<const uint8_t *>(map) + e->offset;
    out->rows = (int)rows;
    out->cols = (int)cols;
    return PINFER_OK;
}

int PqFile::open_file(const char *path) {
    close_file();
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        perror(path);
        return PINFER_E_IO;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 4096) {
        ::close(fd);
        fprintf(stderr, "pinfer (.pq): %s is shorter than a .pq header\n", path);
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
    hdr = static_cast<const PqHeader *>(p);
    int rc = validate_header(*hdr);
    if (rc == PINFER_OK) rc = validate_directory(*this);
    if (rc == PINFER_OK) rc = mat("embed_tokens.weight", hdr->vocab, hdr->hidden, &embed);
    if (rc == PINFER_OK) {
        head = embed;
        if (!hdr->tied_embeddings) rc = mat("lm_head.weight", hdr->vocab, hdr->hidden, &head);
    }
    if (rc == PINFER_OK) rc = vec("norm.weight", hdr->hidden, &norm);
    for (uint32_t i = 0; rc == PINFER_OK && i < hdr->n_layers; i++) {
        char prefix[32];
        snprintf(prefix, sizeof prefix, "layers.%u.", i);
        rc = bind_block(*this, prefix, (hdr->full_attn_mask >> i) & 1, &layers[i]);
    }
    if (rc != PINFER_OK) {
        close_file();
        return rc;
    }
    // The reference maps the MTP head only when a speculative generation first needs it, so a
    // missing or malformed head does not fail the load; generation with k > 0 then returns
    // PINFER_E_FORMAT. The head's decoder block is always a full-attention block.
    if (hdr->has_mtp) {
        const uint32_t H = hdr->hidden;
        const char *vecs[3] = {"mtp.pre_fc_norm_embedding.weight", "mtp.pre_fc_norm_hidden.weight", "mtp.norm.weight"};
        const float **dst[3] = {&mtp.norm_emb, &mtp.norm_hid, &mtp.norm_out};
        bool ok = find("mtp.fc.weight") && mat("mtp.fc.weight", H, 2 * H, &mtp.fc) == PINFER_OK;
        for (int i = 0; i < 3; i++) ok = ok && find(vecs[i]) && vec(vecs[i], H, dst[i]) == PINFER_OK;
        ok = ok && find("mtp.layers.0.self_attn.q_proj.weight") &&
             bind_block(*this, "mtp.layers.0.", true, &mtp.layer) == PINFER_OK;
        mtp.ok = ok;
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

// The model fingerprint that state blobs carry (the reference's pf_model_fingerprint,
// model.c:142-154; it has to be the same number for blobs to move between the engines): 64-bit
// FNV-1a over the header, the directory, and the first, middle and last 64 bytes (or all of it,
// if shorter) of every tensor's data.
uint64_t PqFile::fingerprint() const {
    struct Fnv {
        uint64_t h = 14695981039346656037ull;
        void eat(const void *p, size_t n) {
            const unsigned char *b = static_cast<const unsigned char *>(p);
            for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 1099511628211ull;
        }
    } fnv;
    fnv.eat(hdr, sizeof(PqHeader));
    fnv.eat(dir, (size_t)hdr->n_tensors * sizeof(PqEntry));
    for (uint32_t i = 0; i < hdr->n_tensors; i++) {
        const unsigned char *data = static_cast<const unsigned char *>(map) + dir[i].offset;
        const size_t n = (size_t)dir[i].nbytes, w = n < 64 ? n : 64;
        for (size_t at : {(size_t)0, (n - w) / 2, n - w}) fnv.eat(data + at, w);
    }
    return fnv.h;
}

}  // namespace nb
