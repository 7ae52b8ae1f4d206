/*
 * engine.c - the engine.h interface over the B200 decode path (C11 host).
 *
 * engine_open():
 *   1. maps the GGUF file read-only and parses header, metadata, tensor
 *      directory and data offset with the same acceptance rules as the
 *      reference (src/checkpoint_gguf.c:50-1275, src/config.c:1-54);
 *   2. binds the llama tensors with the reference's shape / type / size
 *      checks (src/gguf_model.c:44-308, incl. the rope_freqs refusal and a
 *      tied output), and its RoPE check (src/gguf_forward.c:107-114);
 *   3. lays the bound tensors out in one device arena (256-byte aligned
 *      starts) and uploads their bytes unchanged;
 *   4. caps the context like src/engine.c:143-162, builds the RoPE cos/sin
 *      table with the same float expressions and libm calls the reference
 *      evaluates per step (src/gguf_forward.c:50-66), loads the vocabulary,
 *      and hands everything to the device side (pk_device.cu), which
 *      allocates the KV cache and captures the decode-step graph.
 * engine_forward() validates (token, pos) on the host and replays the graph.
 */
#define _POSIX_C_SOURCE 200809L
#include "engine.h"
#include "engine_ext.h"
#include "pk_dev.h"

#include <fcntl.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* vocab.c */
int pk_vocab_load_gguf(Tokenizer *t, const unsigned char *file, size_t size, char *err, size_t cap);
int pk_vocab_load_bin(Tokenizer *t, const char *path, size_t vocab_size, char *err, size_t cap);

/* ------------------------------------------------------------------ */
/* GGML type table (a format table shared with every GGUF reader:      */
/* id, name, weights per block, bytes per block)                       */
/* ------------------------------------------------------------------ */

typedef struct {
    uint32_t id;
    const char *name;
    uint32_t block, bytes;
} TypeRow;

static const TypeRow TYPES[] = {
    {0, "F32", 1, 4},        {1, "F16", 1, 2},        {2, "Q4_0", 32, 18},     {3, "Q4_1", 32, 20},
    {6, "Q5_0", 32, 22},     {7, "Q5_1", 32, 24},     {8, "Q8_0", 32, 34},     {9, "Q8_1", 32, 40},
    {10, "Q2_K", 256, 84},   {11, "Q3_K", 256, 110},  {12, "Q4_K", 256, 144},  {13, "Q5_K", 256, 176},
    {14, "Q6_K", 256, 210},  {15, "Q8_K", 256, 292},  {16, "IQ2_XXS", 256, 66}, {17, "IQ2_XS", 256, 74},
    {18, "IQ3_XXS", 256, 98}, {19, "IQ1_S", 256, 50}, {20, "IQ4_NL", 32, 18},  {21, "IQ3_S", 256, 110},
    {22, "IQ2_S", 256, 82},  {23, "IQ4_XS", 256, 136}, {24, "I8", 1, 1},      {25, "I16", 1, 2},
    {26, "I32", 1, 4},       {27, "I64", 1, 8},       {28, "F64", 1, 8},       {29, "IQ1_M", 256, 56},
    {30, "BF16", 1, 2},
};

static const TypeRow *type_row(uint32_t id)
{
    for (size_t i = 0; i < sizeof(TYPES) / sizeof(TYPES[0]); i++) {
        if (TYPES[i].id == id) return &TYPES[i];
    }
    return NULL;
}

static const char *type_name(uint32_t id)
{
    const TypeRow *r = type_row(id);
    return r ? r->name : "UNKNOWN";
}

/* Types the device kernels decode: F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K. */
static int type_supported(uint32_t id)
{
    return id == 0 || id == 1 || id == 2 || id == 8 || id == 12 || id == 13 || id == 14;
}

/* ------------------------------------------------------------------ */
/* Handle                                                              */
/* ------------------------------------------------------------------ */

typedef struct {
    char *name;
    uint32_t ndim, type;
    uint64_t dims[4], offset;
} GTensor;

typedef struct {
    const GTensor *t;
    PkdTensor dev;     /* this rank's slice of the tensor */
    uint64_t r0, c0;   /* its first row and column in the file tensor */
    uint64_t file_rb;  /* bytes per row in the file */
} Bound;

struct LLMModel {
    LLMFormat format;
    Config config;
    int file_context;
    Tokenizer tokenizer;
    char description[256];
    PkdCtx *dev;
    PkbCtx *batch;     /* batched decode state (engine_batch_open), or NULL */
    PkbCtx *prefill;   /* engine_prefill's state (its KV cache is the decode step's), made on first use */
    uint64_t weight_bytes;
    int tp_world;      /* tensor-parallel ranks (1: single GPU) */
    int connected;     /* the decode step exists (tensor parallel: after engine_tp_connect) */
    int batch_seqs;    /* sequences of the batched state */
    int kv_half;       /* KV cache entries in IEEE half (POCKET_CUDA_KV=f16) */
    int kv_head0, kv_heads;  /* this rank's KV heads (all of them on one GPU) */
    int *filled;       /* batched sequences: positions 0 .. filled[s] - 1 hold K/V */
    char last_error[256];
};

static void seterr(char *e, size_t cap, const char *msg)
{
    if (e != NULL && cap > 0) snprintf(e, cap, "%s", msg);
}

/* ------------------------------------------------------------------ */
/* Bounds-checked cursor over the mapped file                          */
/* ------------------------------------------------------------------ */

typedef struct {
    const unsigned char *p;
    size_t n, pos;
    int bad;
} Cur;

static uint64_t rd(Cur *c, int bytes)
{
    if (c->bad || (size_t)bytes > c->n - c->pos) {
        c->bad = 1;
        return 0;
    }
    uint64_t v = 0;
    for (int i = 0; i < bytes; i++) v |= (uint64_t)c->p[c->pos + (size_t)i] << (8 * i);
    c->pos += (size_t)bytes;
    return v;
}

static float rdf(Cur *c)
{
    uint32_t b = (uint32_t)rd(c, 4);
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* GGUF string: u64 length + bytes. Lengths over 1 MiB are refused
 * (src/checkpoint_gguf.c:196-199). */
static const char *rds(Cur *c, uint64_t *len)
{
    *len = rd(c, 8);
    if (c->bad || *len > (1u << 20) || *len > c->n - c->pos) {
        c->bad = 1;
        return NULL;
    }
    const char *s = (const char *)c->p + c->pos;
    c->pos += (size_t)*len;
    return s;
}

static int scalar_size(uint32_t t)
{
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

static void skip_value(Cur *c, uint32_t t)
{
    uint64_t len;
    if (t == 8) {
        (void)rds(c, &len);
    } else if (t == 9) {
        uint32_t et = (uint32_t)rd(c, 4);
        uint64_t n = rd(c, 8);
        if (et > 12 || et == 9) {
            c->bad = 1;
            return;
        }
        for (uint64_t i = 0; i < n && !c->bad; i++) skip_value(c, et);
    } else {
        int s = scalar_size(t);
        if (s == 0 || (size_t)s > c->n - c->pos) {
            c->bad = 1;
            return;
        }
        c->pos += (size_t)s;
    }
}

static int is_key(const char *k, uint64_t n, const char *s)
{
    return strlen(s) == n && memcmp(k, s, (size_t)n) == 0;
}

typedef struct {
    const unsigned char *map;
    size_t size;
    Config c;
    GTensor *t;
    size_t nt;
    uint64_t data_off;
} Parsed;

static void parsed_free(Parsed *p)
{
    if (p->t) {
        for (size_t i = 0; i < p->nt; i++) free(p->t[i].name);
        free(p->t);
    }
    p->t = NULL;
}

/* Config rules of src/config.c:9-50. */
static int config_ok(const Config *c)
{
    if (c->dim <= 0 || c->hidden_dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
        c->vocab_size <= 0 || c->seq_len <= 0)
        return 0;
    if (c->n_kv_heads > c->n_heads || c->n_heads % c->n_kv_heads != 0) return 0;
    if (c->dim % c->n_heads != 0 || (c->dim / c->n_heads) % 2 != 0) return 0;
    return 1;
}

/* Header, metadata and tensor directory (src/checkpoint_gguf.c:50-1030). */
static int parse(Parsed *p, char *err, size_t cap)
{
    Cur c = {p->map, p->size, 0, 0};
    if (p->size < 4 || memcmp(p->map, "GGUF", 4) != 0) {
        seterr(err, cap, "Invalid GGUF magic number.");
        return 0;
    }
    c.pos = 4;
    uint32_t ver = (uint32_t)rd(&c, 4);
    if (c.bad) {
        seterr(err, cap, "Cannot read GGUF version.");
        return 0;
    }
    if (ver == 1) {
        seterr(err, cap, "GGUF version 1 is not supported (use a v2/v3 file).");
        return 0;
    }
    if (ver < 2 || ver > 3) {
        seterr(err, cap, "Unsupported GGUF version.");
        return 0;
    }
    const uint64_t nt = rd(&c, 8), nkv = rd(&c, 8);
    if (c.bad) {
        seterr(err, cap, "Invalid or truncated GGUF metadata.");
        return 0;
    }

    enum { ARCH = 1, DIM = 2, HID = 4, LAY = 8, HEADS = 16, KV = 32, CTX = 64, VOC = 128 };
    unsigned seen = 0;
    Config k;
    memset(&k, 0, sizeof(k));
    char scal_type[32] = "";
    float scal_factor = 0.0f, scal_old = 0.0f;
    uint32_t align = 32;
    const char *bad_meta = "Invalid or unsupported GGUF metadata.";

    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        const char *key = rds(&c, &kl);
        const uint32_t t = (uint32_t)rd(&c, 4);
        if (c.bad) {
            seterr(err, cap, bad_meta);
            return 0;
        }
        if (is_key(key, kl, "general.architecture")) {
            uint64_t al;
            const char *a = t == 8 ? rds(&c, &al) : NULL;
            if (a == NULL) {
                seterr(err, cap, bad_meta);
                return 0;
            }
            if (!(al == 5 && memcmp(a, "llama", 5) == 0)) {
                seterr(err, cap, "Only llama architecture is supported.");
                return 0;
            }
            seen |= ARCH;
        } else if (is_key(key, kl, "tokenizer.ggml.tokens")) {
            if (t != 9) {
                seterr(err, cap, bad_meta);
                return 0;
            }
            uint32_t et = (uint32_t)rd(&c, 4);
            uint64_t n = rd(&c, 8);
            if (c.bad || et != 8 || n == 0 || n > 0x7FFFFFFFull) {
                seterr(err, cap, bad_meta);
                return 0;
            }
            for (uint64_t j = 0; j < n && !c.bad; j++) skip_value(&c, 8);
            k.vocab_size = (int)n;
            seen |= VOC;
        } else if (is_key(key, kl, "llama.rope.freq_base") ||
                   is_key(key, kl, "llama.attention.layer_norm_rms_epsilon") ||
                   is_key(key, kl, "llama.rope.scaling.factor") || is_key(key, kl, "llama.rope.scale_linear")) {
            const float v = t == 6 ? rdf(&c) : NAN;
            if (c.bad || !isfinite(v) || v <= 0.0f) {
                seterr(err, cap, bad_meta);
                return 0;
            }
            if (is_key(key, kl, "llama.rope.freq_base")) k.rope_freq_base = v;
            else if (is_key(key, kl, "llama.attention.layer_norm_rms_epsilon")) k.rms_norm_eps = v;
            else if (is_key(key, kl, "llama.rope.scaling.factor")) scal_factor = v;
            else scal_old = v;
        } else if (is_key(key, kl, "llama.rope.scaling.type")) {
            uint64_t sl;
            const char *s = t == 8 ? rds(&c, &sl) : NULL;
            if (s == NULL) {
                seterr(err, cap, bad_meta);
                return 0;
            }
            snprintf(scal_type, sizeof(scal_type), "%.*s", (int)(sl < 31 ? sl : 31), s);
        } else if (is_key(key, kl, "general.alignment")) {
            const uint32_t v = t == 4 ? (uint32_t)rd(&c, 4) : 0;
            if (c.bad || v == 0 || (v & (v - 1)) != 0) {
                seterr(err, cap, "Cannot determine GGUF tensor data location.");
                return 0;
            }
            align = v;
        } else {
            int *dst = NULL;
            unsigned flag = 0;
            if (is_key(key, kl, "llama.embedding_length")) { dst = &k.dim; flag = DIM; }
            else if (is_key(key, kl, "llama.feed_forward_length")) { dst = &k.hidden_dim; flag = HID; }
            else if (is_key(key, kl, "llama.block_count")) { dst = &k.n_layers; flag = LAY; }
            else if (is_key(key, kl, "llama.attention.head_count")) { dst = &k.n_heads; flag = HEADS; }
            else if (is_key(key, kl, "llama.attention.head_count_kv")) { dst = &k.n_kv_heads; flag = KV; }
            else if (is_key(key, kl, "llama.context_length")) { dst = &k.seq_len; flag = CTX; }
            else if (is_key(key, kl, "llama.rope.dimension_count")) { dst = &k.rope_dim; flag = 0; }
            if (dst != NULL) {
                const uint32_t v = t == 4 ? (uint32_t)rd(&c, 4) : 0;
                if (c.bad || v == 0 || v > 0x7FFFFFFFu) {
                    seterr(err, cap, bad_meta);
                    return 0;
                }
                *dst = (int)v;
                seen |= flag;
            } else {
                skip_value(&c, t);
            }
        }
        if (c.bad) {
            seterr(err, cap, bad_meta);
            return 0;
        }
    }
    if (seen != 0xFFu) {
        seterr(err, cap, "Required LLaMA metadata is missing.");
        return 0;
    }
    /* Defaults and RoPE scaling, src/checkpoint_gguf.c:694-737. */
    if (k.rope_dim == 0) k.rope_dim = k.dim / k.n_heads;
    if (k.rope_freq_base == 0.0f) k.rope_freq_base = 10000.0f;
    if (k.rms_norm_eps == 0.0f) k.rms_norm_eps = 1e-5f;
    k.rope_scale = 1.0f;
    if (scal_type[0] == '\0' || strcmp(scal_type, "none") == 0) {
        if (scal_old > 0.0f) k.rope_scale = scal_old;
        else if (scal_type[0] == '\0' && scal_factor > 0.0f) k.rope_scale = scal_factor;
    } else if (strcmp(scal_type, "linear") == 0) {
        k.rope_scale = scal_factor > 0.0f ? scal_factor : 1.0f;
    } else {
        if (err && cap) {
            snprintf(err, cap, "RoPE scaling type '%s' is not supported (only 'none' and 'linear').", scal_type);
        }
        return 0;
    }
    if (!config_ok(&k)) {
        seterr(err, cap, "Invalid LLaMA model configuration.");
        return 0;
    }

    /* Tensor directory. */
    if (nt > (uint64_t)(SIZE_MAX / sizeof(GTensor)) || nt > p->size) {
        seterr(err, cap, "Too many GGUF tensors.");
        return 0;
    }
    p->t = (GTensor *)calloc(nt ? (size_t)nt : 1, sizeof(GTensor));
    p->nt = (size_t)nt;
    if (p->t == NULL) {
        seterr(err, cap, "Cannot allocate tensor information.");
        return 0;
    }
    for (size_t i = 0; i < p->nt; i++) {
        uint64_t nl;
        const char *nm = rds(&c, &nl);
        const uint32_t nd = (uint32_t)rd(&c, 4);
        if (c.bad || nd == 0 || nd > 4) {
            seterr(err, cap, "Invalid or truncated GGUF tensor information.");
            return 0;
        }
        p->t[i].name = (char *)malloc((size_t)nl + 1);
        if (p->t[i].name == NULL) {
            seterr(err, cap, "Cannot allocate tensor information.");
            return 0;
        }
        memcpy(p->t[i].name, nm, (size_t)nl);
        p->t[i].name[nl] = '\0';
        p->t[i].ndim = nd;
        for (uint32_t d = 0; d < nd; d++) p->t[i].dims[d] = rd(&c, 8);
        p->t[i].type = (uint32_t)rd(&c, 4);
        p->t[i].offset = rd(&c, 8);
        if (c.bad || p->t[i].type > 40) {
            seterr(err, cap, "Invalid or truncated GGUF tensor information.");
            return 0;
        }
    }
    p->data_off = ((uint64_t)c.pos + align - 1) / align * align;
    p->c = k;
    return 1;
}

static const GTensor *find(const Parsed *p, const char *name)
{
    for (size_t i = 0; i < p->nt; i++) {
        if (strcmp(p->t[i].name, name) == 0) return &p->t[i];
    }
    return NULL;
}

/* bind_weight, src/gguf_model.c:44-128. rows == 0: a 1-D tensor. */
static int bind(const Parsed *p, const char *name, uint64_t cols, uint64_t rows, Bound *b, char *err,
                size_t cap)
{
    const GTensor *t = find(p, name);
    if (t == NULL) {
        if (err && cap) snprintf(err, cap, "Missing tensor: %s", name);
        return 0;
    }
    const uint32_t nd = rows == 0 ? 1u : 2u;
    const uint64_t nr = rows == 0 ? 1u : rows;
    if (t->ndim != nd || t->dims[0] != cols || (nd == 2 && t->dims[1] != rows)) {
        if (err && cap) snprintf(err, cap, "Tensor %s has an unexpected shape.", name);
        return 0;
    }
    if (!type_supported(t->type)) {
        if (err && cap) snprintf(err, cap, "Tensor %s uses unsupported type %s (%u).", name, type_name(t->type), t->type);
        return 0;
    }
    const TypeRow *tr = type_row(t->type);
    /* Storage size from the directory (src/checkpoint_gguf.c:1175-1225). */
    uint64_t elems = 1;
    for (uint32_t d = 0; d < t->ndim; d++) {
        if (t->dims[d] == 0 || elems > UINT64_MAX / t->dims[d]) {
            if (err && cap) snprintf(err, cap, "Tensor %s lies outside the file.", name);
            return 0;
        }
        elems *= t->dims[d];
    }
    if (t->dims[0] % tr->block || elems % tr->block) {
        if (err && cap) snprintf(err, cap, "Tensor %s lies outside the file.", name);
        return 0;
    }
    const uint64_t size = elems / tr->block * tr->bytes;
    const uint64_t off = p->data_off + t->offset;
    if (t->offset > UINT64_MAX - p->data_off || off > p->size || size > p->size - off) {
        if (err && cap) snprintf(err, cap, "Tensor %s lies outside the file.", name);
        return 0;
    }
    if (cols % tr->block) {
        seterr(err, cap, "Invalid row layout.");
        return 0;
    }
    const uint64_t rb = cols / tr->block * tr->bytes;
    if (rb * nr != size) {
        if (err && cap) snprintf(err, cap, "Tensor %s: storage size does not match its shape.", name);
        return 0;
    }
    b->t = t;
    b->dev.type = t->type;
    b->dev.rows = nr;
    b->dev.cols = cols;
    b->dev.row_bytes = rb;
    b->r0 = 0;
    b->c0 = 0;
    b->file_rb = rb;
    return 1;
}

/* Keep rows [r0, r0 + nr) and columns [c0, c0 + nc) of a bound tensor
 * (columns on whole quant blocks). */
static void slice(Bound *b, uint64_t r0, uint64_t nr, uint64_t c0, uint64_t nc)
{
    const TypeRow *tr = type_row(b->dev.type);
    b->r0 = r0;
    b->c0 = c0;
    b->dev.rows = nr;
    b->dev.cols = nc;
    b->dev.row_bytes = nc / tr->block * tr->bytes;
}

/* Tensor-parallel placement (see EngineTpPlan in engine_ext.h). */
static int tp_plan(int dim, int hid, int nh, int nkv, int voc, int wo_bw, int dn_bw, int rank, int world, PkdTp *t,
                   char *err, size_t cap)
{
    memset(t, 0, sizeof(*t));
    if (world < 1 || world > PKD_TP_MAX || rank < 0 || rank >= world) {
        seterr(err, cap, "Tensor-parallel world must be 1..8 with 0 <= rank < world.");
        return 0;
    }
    if (dim <= 0 || hid <= 0 || nh <= 0 || nkv <= 0 || voc <= 0 || wo_bw <= 0 || dn_bw <= 0 || dim % nh ||
        nh % nkv) {
        seterr(err, cap, "Invalid model dimensions.");
        return 0;
    }
    if (nh % world) {
        if (err && cap) snprintf(err, cap, "%d attention heads cannot be split over %d ranks.", nh, world);
        return 0;
    }
    const int hs = dim / nh, kvm = nh / nkv;
    t->rank = rank;
    t->world = world;
    t->q_heads = nh / world;
    t->q_head0 = rank * t->q_heads;
    if (nkv % world == 0) {
        t->kv_heads = nkv / world;
        t->kv_head0 = rank * t->kv_heads;
    } else if (world % nkv == 0 && kvm % (world / nkv) == 0) {
        t->kv_heads = 1;  /* ranks share a KV head; each computes it */
        t->kv_head0 = t->q_head0 / kvm;
    } else {
        if (err && cap) snprintf(err, cap, "%d KV heads cannot be split over %d ranks.", nkv, world);
        return 0;
    }
    if ((t->q_heads * hs) % wo_bw) {
        seterr(err, cap, "attn_output quant blocks straddle the head split.");
        return 0;
    }
    if (hid % dn_bw || hid / dn_bw < world) {
        seterr(err, cap, "ffn_down has fewer quant blocks than ranks.");
        return 0;
    }
    const long nb = hid / dn_bw;
    for (int r = 0; r < world; r++) {
        const int h0 = (int)(dn_bw * (nb * r / world)), h1 = (int)(dn_bw * (nb * (r + 1) / world));
        if (h1 - h0 > t->hid_max) t->hid_max = h1 - h0;
        if (r == rank) {
            t->hid0 = h0;
            t->hid = h1 - h0;
        }
        t->own0[r] = (int)((long)dim * r / world);
        t->own[r] = (int)((long)dim * (r + 1) / world) - t->own0[r];
        if (t->own[r] > t->own_max) t->own_max = t->own[r];
    }
    t->voc0 = (int)((long)voc * rank / world);
    t->voc = (int)((long)voc * (rank + 1) / world) - t->voc0;
    return 1;
}

int engine_tp_plan(int dim, int hidden_dim, int n_heads, int n_kv_heads, int vocab_size, int wo_block,
                   int down_block, int rank, int world, EngineTpPlan *out, char *err, size_t cap)
{
    PkdTp t;
    if (out == NULL) {
        seterr(err, cap, "No output given.");
        return 0;
    }
    if (!tp_plan(dim, hidden_dim, n_heads, n_kv_heads, vocab_size, wo_block, down_block, rank, world, &t, err,
                 cap))
        return 0;
    out->q_head0 = t.q_head0;
    out->q_heads = t.q_heads;
    out->kv_head0 = t.kv_head0;
    out->kv_heads = t.kv_heads;
    out->hid0 = t.hid0;
    out->hid = t.hid;
    out->voc0 = t.voc0;
    out->voc = t.voc;
    out->own0 = t.own0[rank];
    out->own = t.own[rank];
    if (err && cap) err[0] = '\0';
    return 1;
}

/* "GGUF, weights Q4_K x135 Q6_K x21 F32 x45", src/engine.c:95-117 (counts
 * of every tensor in the file, by type id order). */
static void describe(LLMModel *m, const Parsed *p)
{
    unsigned counts[64] = {0};
    size_t used = (size_t)snprintf(m->description, sizeof(m->description), "GGUF, weights");
    for (size_t i = 0; i < p->nt; i++) {
        if (p->t[i].type < 64) counts[p->t[i].type]++;
    }
    for (uint32_t t = 0; t < 64 && used < sizeof(m->description); t++) {
        if (counts[t]) {
            used += (size_t)snprintf(m->description + used, sizeof(m->description) - used, " %s x%u",
                                     type_name(t), counts[t]);
        }
    }
}

static int env_device(void)
{
    const char *s = getenv("POCKET_CUDA_DEVICE");
    return (s != NULL && *s) ? atoi(s) : 0;
}

/* KV cache entry type from POCKET_CUDA_KV: unset, "" or "f32" -> float (0),
 * "f16" -> IEEE half (1), anything else -> -1 (the open fails). */
static int env_kv_half(void)
{
    const char *s = getenv("POCKET_CUDA_KV");
    if (s == NULL || *s == '\0' || strcmp(s, "f32") == 0) return 0;
    if (strcmp(s, "f16") == 0) return 1;
    return -1;
}

void engine_close(LLMModel *m)
{
    if (m == NULL) return;
    tokenizer_free(&m->tokenizer);
    pkb_destroy(m->batch);
    pkb_destroy(m->prefill);
    free(m->filled);
    pkd_destroy(m->dev);
    free(m);
}

static LLMModel *open_impl(const LLMOptions *o, int device, int rank, int world, char *err, size_t cap)
{
    if (o == NULL || o->model_path == NULL || o->model_path[0] == '\0') {
        seterr(err, cap, "No model path given.");
        return NULL;
    }
    if (o->max_context < 0) {
        seterr(err, cap, "Context size must be positive.");
        return NULL;
    }
    const int kv_half = env_kv_half();
    if (kv_half < 0) {
        seterr(err, cap, "POCKET_CUDA_KV must be f32 or f16.");
        return NULL;
    }
    const int fd = open(o->model_path, O_RDONLY);
    if (fd == -1) {
        seterr(err, cap, "Cannot open model file.");
        return NULL;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        seterr(err, cap, "Cannot open model file.");
        return NULL;
    }
    Parsed p;
    memset(&p, 0, sizeof(p));
    p.size = (size_t)st.st_size;
    void *map = mmap(NULL, p.size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) {
        seterr(err, cap, "Cannot memory-map GGUF file.");
        return NULL;
    }
    p.map = (const unsigned char *)map;
    if (p.size < 4 || memcmp(p.map, "GGUF", 4) != 0) {
        munmap(map, p.size);
        seterr(err, cap, "Not a GGUF file: this engine runs quantized GGUF models only.");
        return NULL;
    }

    LLMModel *m = (LLMModel *)calloc(1, sizeof(LLMModel));
    Bound *b = NULL;
    PkdTensor *lt = NULL;
    float *rope = NULL;
    if (m == NULL) {
        munmap(map, p.size);
        seterr(err, cap, "Out of memory.");
        return NULL;
    }
    m->format = LLM_FORMAT_GGUF;
    m->kv_half = kv_half;
    if (!parse(&p, err, cap)) goto fail;
    if (find(&p, "rope_freqs.weight") != NULL) {
        seterr(err, cap, "Model uses RoPE frequency factors (rope_freqs.weight, Llama 3.1 style), which are not supported.");
        goto fail;
    }
    {
        Config *c = &p.c;
        const uint64_t dim = (uint64_t)c->dim, hid = (uint64_t)c->hidden_dim, voc = (uint64_t)c->vocab_size;
        const uint64_t hs = dim / (uint64_t)c->n_heads, kvd = hs * (uint64_t)c->n_kv_heads;
        const int L = c->n_layers;
        /* bound: 0 embd, 1 output_norm, 2 output, then 9 per layer */
        const size_t nb = 3 + 9 * (size_t)L;
        b = (Bound *)calloc(nb, sizeof(Bound));
        lt = (PkdTensor *)calloc(9 * (size_t)L, sizeof(PkdTensor));
        if (b == NULL || lt == NULL) {
            seterr(err, cap, "Out of memory.");
            goto fail;
        }
        if (!bind(&p, "token_embd.weight", dim, voc, &b[0], err, cap) ||
            !bind(&p, "output_norm.weight", dim, 0, &b[1], err, cap))
            goto fail;
        if (find(&p, "output.weight") == NULL) {
            b[2] = b[0]; /* tied output, src/gguf_model.c:257-266 */
        } else if (!bind(&p, "output.weight", dim, voc, &b[2], err, cap)) {
            goto fail;
        }
        static const char *suffix[9] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight",
                                        "attn_v.weight", "attn_output.weight", "ffn_norm.weight",
                                        "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
        const uint64_t cols[9] = {dim, dim, dim, dim, dim, dim, dim, dim, hid};
        const uint64_t rows[9] = {0, dim, kvd, kvd, dim, 0, hid, hid, dim};
        for (int l = 0; l < L; l++) {
            for (int j = 0; j < 9; j++) {
                char nm[96];
                snprintf(nm, sizeof(nm), "blk.%d.%s", l, suffix[j]);
                if (!bind(&p, nm, cols[j], rows[j], &b[3 + 9 * (size_t)l + (size_t)j], err, cap)) goto fail;
            }
        }
        /* src/gguf_forward.c:107-114 */
        if (c->rope_dim <= 0 || c->rope_dim % 2 != 0 || (uint64_t)c->rope_dim > hs || !(c->rope_scale > 0.0f)) {
            seterr(err, cap, "Unsupported RoPE dimension.");
            goto fail;
        }
        /* This rank's slices (world 1: every tensor whole). The block
         * widths that bound the column splits are the widest over layers. */
        int wo_bw = 1, dn_bw = 1;
        for (int l = 0; l < L; l++) {
            const int w1 = (int)type_row(b[3 + 9 * (size_t)l + 4].dev.type)->block;
            const int w2 = (int)type_row(b[3 + 9 * (size_t)l + 8].dev.type)->block;
            if (w1 > wo_bw) wo_bw = w1;
            if (w2 > dn_bw) dn_bw = w2;
        }
        PkdTp tp;
        if (!tp_plan(c->dim, c->hidden_dim, c->n_heads, c->n_kv_heads, c->vocab_size, wo_bw, dn_bw, rank, world,
                     &tp, err, cap))
            goto fail;
        const int tied = b[2].t == b[0].t;
        if (world > 1) {
            const uint64_t qr0 = (uint64_t)tp.q_head0 * hs, qn = (uint64_t)tp.q_heads * hs;
            const uint64_t kr0 = (uint64_t)tp.kv_head0 * hs, kn = (uint64_t)tp.kv_heads * hs;
            slice(&b[2], (uint64_t)tp.voc0, (uint64_t)tp.voc, 0, dim);
            for (int l = 0; l < L; l++) {
                Bound *lb = b + 3 + 9 * (size_t)l;
                slice(&lb[1], qr0, qn, 0, dim);                               /* wq rows */
                slice(&lb[2], kr0, kn, 0, dim);                               /* wk rows */
                slice(&lb[3], kr0, kn, 0, dim);                               /* wv rows */
                slice(&lb[4], 0, dim, qr0, qn);                               /* wo columns */
                slice(&lb[6], (uint64_t)tp.hid0, (uint64_t)tp.hid, 0, dim);   /* gate rows */
                slice(&lb[7], (uint64_t)tp.hid0, (uint64_t)tp.hid, 0, dim);   /* up rows */
                slice(&lb[8], 0, dim, (uint64_t)tp.hid0, (uint64_t)tp.hid);   /* down columns */
            }
        }
        /* Arena layout; a whole tied output shares the embedding bytes. */
        uint64_t arena = 0;
        for (size_t i = 0; i < nb; i++) {
            if (i == 2 && tied && world == 1) {
                b[2].dev.offset = b[0].dev.offset;
                continue;
            }
            b[i].dev.offset = arena;
            arena += (b[i].dev.rows * b[i].dev.row_bytes + 255) / 256 * 256;
        }
        m->weight_bytes = arena;

        /* Context cap, src/engine.c:143-162. */
        m->file_context = c->seq_len;
        int ctx = o->max_context;
        if (ctx <= 0) ctx = c->seq_len < LLM_DEFAULT_MAX_CONTEXT ? c->seq_len : LLM_DEFAULT_MAX_CONTEXT;
        if (ctx > c->seq_len) ctx = c->seq_len;
        c->seq_len = ctx;
        m->config = *c;

        /* Vocabulary (src/engine.c:276-285). */
        const int rc = o->tokenizer_path != NULL
                           ? pk_vocab_load_bin(&m->tokenizer, o->tokenizer_path, (size_t)c->vocab_size, err, cap)
                           : pk_vocab_load_gguf(&m->tokenizer, p.map, p.size, err, cap);
        if (rc != 0) goto fail;

        /* RoPE table: the values rope_head() computes at each position,
         * same float expressions, same libm (src/gguf_forward.c:50-66). */
        const size_t rd2 = (size_t)c->rope_dim;
        rope = (float *)malloc((size_t)ctx * rd2 * sizeof(float) + sizeof(float));
        float *freq = (float *)malloc(rd2 * sizeof(float));
        if (rope == NULL || freq == NULL) {
            free(freq);
            seterr(err, cap, "Out of memory.");
            goto fail;
        }
        for (int i = 0; i < c->rope_dim; i += 2) {
            freq[i] = 1.0f / powf(c->rope_freq_base, (float)i / (float)c->rope_dim);
        }
        for (int pos = 0; pos < ctx; pos++) {
            const float position = (float)pos / c->rope_scale;
            for (int i = 0; i < c->rope_dim; i += 2) {
                const float angle = position * freq[i];
                rope[(size_t)pos * rd2 + (size_t)i] = cosf(angle);
                rope[(size_t)pos * rd2 + (size_t)i + 1] = sinf(angle);
            }
        }
        free(freq);

        /* Device: upload, run state, graph. */
        m->dev = pkd_create(device, arena, err, cap);
        if (m->dev == NULL) goto fail;
        for (size_t i = 0; i < nb; i++) {
            if (i == 2 && tied && world == 1) continue;
            const Bound *bi = &b[i];
            const unsigned char *src = p.map + p.data_off + bi->t->offset + bi->r0 * bi->file_rb;
            const uint64_t bytes = bi->dev.rows * bi->dev.row_bytes;
            if (bi->dev.row_bytes == bi->file_rb) {  /* whole rows: one contiguous range */
                if (!pkd_upload(m->dev, bi->dev.offset, src, bytes, err, cap)) goto fail;
                continue;
            }
            /* a column slice: gather each row's byte range */
            const TypeRow *tr = type_row(bi->dev.type);
            const uint64_t cb = bi->c0 / tr->block * tr->bytes;
            unsigned char *tmp = (unsigned char *)malloc((size_t)bytes);
            if (tmp == NULL) {
                seterr(err, cap, "Out of memory.");
                goto fail;
            }
            for (uint64_t r = 0; r < bi->dev.rows; r++) {
                memcpy(tmp + r * bi->dev.row_bytes, src + r * bi->file_rb + cb, (size_t)bi->dev.row_bytes);
            }
            const int ok = pkd_upload(m->dev, bi->dev.offset, tmp, bytes, err, cap);
            free(tmp);
            if (!ok) goto fail;
        }
        PkdModel dm;
        memset(&dm, 0, sizeof(dm));
        dm.dim = c->dim;
        dm.hidden_dim = tp.hid;
        dm.n_layers = L;
        dm.n_heads = tp.q_heads;
        dm.n_kv_heads = tp.kv_heads;
        dm.head_size = (int)hs;
        dm.tp = tp;
        m->kv_head0 = tp.kv_head0;
        m->kv_heads = tp.kv_heads;
        dm.vocab_size = c->vocab_size;
        dm.seq_len = ctx;
        dm.rope_dim = c->rope_dim;
        dm.rms_eps = c->rms_norm_eps;
        dm.att_scale = 1.0f / sqrtf((float)hs);
        dm.kv_half = m->kv_half;
        dm.embd = b[0].dev;
        dm.output_norm = b[1].dev;
        dm.output = b[2].dev;
        PkdTensor *an = lt, *wq = lt + L, *wk = lt + 2 * L, *wv = lt + 3 * L, *wo = lt + 4 * L;
        PkdTensor *fn = lt + 5 * L, *gt = lt + 6 * L, *up = lt + 7 * L, *dn = lt + 8 * L;
        for (int l = 0; l < L; l++) {
            const Bound *lb = b + 3 + 9 * (size_t)l;
            an[l] = lb[0].dev;
            wq[l] = lb[1].dev;
            wk[l] = lb[2].dev;
            wv[l] = lb[3].dev;
            wo[l] = lb[4].dev;
            fn[l] = lb[5].dev;
            gt[l] = lb[6].dev;
            up[l] = lb[7].dev;
            dn[l] = lb[8].dev;
        }
        dm.attn_norm = an;
        dm.ffn_norm = fn;
        dm.wq = wq;
        dm.wk = wk;
        dm.wv = wv;
        dm.wo = wo;
        dm.gate = gt;
        dm.up = up;
        dm.down = dn;
        dm.rope_cs = rope;
        if (!pkd_build(m->dev, &dm, err, cap)) goto fail;
        m->tp_world = world;
        m->connected = world == 1;
        describe(m, &p);
    }
    free(rope);
    free(b);
    free(lt);
    parsed_free(&p);
    munmap(map, p.size);
    if (err && cap) err[0] = '\0';
    return m;

fail:
    free(rope);
    free(b);
    free(lt);
    parsed_free(&p);
    munmap(map, p.size);
    engine_close(m);
    return NULL;
}

LLMModel *engine_open_device(const LLMOptions *o, int device, char *err, size_t cap)
{
    return open_impl(o, device, 0, 1, err, cap);
}

LLMModel *engine_open_tp(const LLMOptions *o, int device, int rank, int world, char *err, size_t cap)
{
    return open_impl(o, device, rank, world, err, cap);
}

int engine_tp_handle(LLMModel *m, void *out64)
{
    if (m == NULL || m->tp_world < 2 || out64 == NULL) return 0;
    return pkd_tp_handle(m->dev, out64, m->last_error, sizeof(m->last_error));
}

int engine_tp_connect(LLMModel *m, const void *handles, char *err, size_t cap)
{
    if (m == NULL || m->tp_world < 2 || handles == NULL || m->connected) {
        seterr(err, cap, "Not a tensor-parallel handle waiting to be connected.");
        return 0;
    }
    if (!pkd_tp_connect(m->dev, handles, err, cap)) {
        snprintf(m->last_error, sizeof(m->last_error), "%s", err != NULL && cap > 0 ? err : "connect failed");
        return 0;
    }
    m->connected = 1;
    if (err && cap) err[0] = '\0';
    return 1;
}

LLMModel *engine_open(const LLMOptions *o, char *err, size_t cap)
{
    return engine_open_device(o, env_device(), err, cap);
}

static int step_ok(const LLMModel *m, int token, int pos)
{
    return m != NULL && m->dev != NULL && m->connected && token >= 0 && token < m->config.vocab_size && pos >= 0 &&
           pos < m->config.seq_len;
}

float *engine_forward(LLMModel *m, int token, int pos)
{
    if (!step_ok(m, token, pos)) return NULL;
    float *r = pkd_forward(m->dev, token, pos);
    if (r == NULL) snprintf(m->last_error, sizeof(m->last_error), "%s", pkd_error(m->dev));
    return r;
}

int engine_forward_greedy(LLMModel *m, int token, int pos)
{
    if (!step_ok(m, token, pos)) return -2;
    const int r = pkd_forward_greedy(m->dev, token, pos);
    if (r == -2) snprintf(m->last_error, sizeof(m->last_error), "%s", pkd_error(m->dev));
    return r;
}

int engine_generate_greedy(LLMModel *m, int token, int pos, int n, int *out_tokens, float *device_ms)
{
    if (!step_ok(m, token, pos) || n < 0 || n > m->config.seq_len - pos || (n > 0 && out_tokens == NULL)) {
        return 0;
    }
    if (!pkd_generate_greedy(m->dev, token, pos, n, out_tokens, device_ms)) {
        snprintf(m->last_error, sizeof(m->last_error), "%s", pkd_error(m->dev));
        return 0;
    }
    return 1;
}

int engine_batch_open(LLMModel *m, int max_seqs, char *err, size_t cap)
{
    if (m == NULL || m->dev == NULL || !m->connected) {
        seterr(err, cap, "No model.");
        return 0;
    }
    if (max_seqs < 1 || max_seqs > ENGINE_BATCH_MAX) {
        seterr(err, cap, "Batched decode takes 1 to 64 sequences.");
        return 0;
    }
    pkb_destroy(m->batch);  /* a new open drops the old sequences */
    m->batch = NULL;
    free(m->filled);
    m->filled = (int *)calloc((size_t)max_seqs, sizeof(int));
    if (m->filled == NULL) {
        seterr(err, cap, "Out of memory.");
        return 0;
    }
    m->batch = pkb_create(m->dev, max_seqs, err, cap);
    if (m->batch == NULL) return 0;
    m->batch_seqs = max_seqs;
    if (err && cap) err[0] = '\0';
    return 1;
}

int engine_forward_batch(LLMModel *m, const int *tokens, const int *pos, const int *seq_ids, int n,
                         int *next_tokens, float *logits)
{
    if (m == NULL || m->batch == NULL || tokens == NULL || pos == NULL || seq_ids == NULL || next_tokens == NULL ||
        n < 1 || n > ENGINE_BATCH_MAX)
        return 0;
    for (int i = 0; i < n; i++) {
        if (tokens[i] < 0 || tokens[i] >= m->config.vocab_size || pos[i] < 0 || pos[i] >= m->config.seq_len ||
            seq_ids[i] < 0 || seq_ids[i] >= m->batch_seqs)
            return 0;
        for (int j = 0; j < i; j++)  /* each (sequence, position) once per step */
            if (seq_ids[j] == seq_ids[i] && pos[j] == pos[i]) return 0;
    }
    /* No gaps: a row at position p of sequence s needs K/V at 0 .. p - 1,
     * from earlier steps (filled[s]) or from rows of this call (every
     * position in [filled[s], p) among them). */
    for (int i = 0; i < n; i++) {
        const int s0 = seq_ids[i], f = m->filled[s0];
        if (pos[i] <= f) continue;
        int have = 0;
        for (int j = 0; j < n; j++)
            if (seq_ids[j] == s0 && pos[j] >= f && pos[j] < pos[i]) have++;
        if (have != pos[i] - f) {
            snprintf(m->last_error, sizeof(m->last_error),
                     "Sequence %d has no K/V at positions %d .. %d (row at position %d).", s0, f, pos[i] - 1,
                     pos[i]);
            return 0;
        }
    }
    if (!pkb_step(m->batch, tokens, pos, seq_ids, n, next_tokens, logits)) {
        snprintf(m->last_error, sizeof(m->last_error), "%s", pkb_error(m->batch));
        return 0;
    }
    for (int i = 0; i < n; i++)
        if (pos[i] + 1 > m->filled[seq_ids[i]]) m->filled[seq_ids[i]] = pos[i] + 1;
    return 1;
}

int engine_prefill(LLMModel *m, const int *tokens, int n, int pos0, float *last_logits, char *err, size_t cap)
{
    if (m == NULL || m->dev == NULL || !m->connected || tokens == NULL || n < 1 || pos0 < 0 ||
        pos0 > m->config.seq_len - n) {
        seterr(err, cap, "Invalid arguments.");
        return -2;
    }
    for (int i = 0; i < n; i++) {
        if (tokens[i] < 0 || tokens[i] >= m->config.vocab_size) {
            seterr(err, cap, "Token outside the vocabulary.");
            return -2;
        }
    }
    if (m->prefill == NULL) {
        m->prefill = pkb_create_prefill(m->dev, err, cap);
        if (m->prefill == NULL) return -2;
    }
    int pos[ENGINE_BATCH_MAX], seq[ENGINE_BATCH_MAX], next[ENGINE_BATCH_MAX];
    float *lg = NULL;
    int last = -2;
    for (int i0 = 0; i0 < n; i0 += ENGINE_BATCH_MAX) {
        const int k = n - i0 < ENGINE_BATCH_MAX ? n - i0 : ENGINE_BATCH_MAX;
        const int final = i0 + k == n;
        for (int j = 0; j < k; j++) {
            pos[j] = pos0 + i0 + j;
            seq[j] = 0;
        }
        if (final && last_logits != NULL) {
            lg = (float *)malloc((size_t)k * (size_t)m->config.vocab_size * sizeof(float));
            if (lg == NULL) {
                seterr(err, cap, "Out of memory.");
                return -2;
            }
        }
        if (!pkb_step(m->prefill, tokens + i0, pos, seq, k, next, final ? lg : NULL)) {
            snprintf(m->last_error, sizeof(m->last_error), "%s", pkb_error(m->prefill));
            seterr(err, cap, m->last_error);
            free(lg);
            return -2;
        }
        if (final) {
            last = next[k - 1];
            if (lg != NULL)
                memcpy(last_logits, lg + (size_t)(k - 1) * m->config.vocab_size,
                       (size_t)m->config.vocab_size * sizeof(float));
        }
    }
    free(lg);
    if (err && cap) err[0] = '\0';
    return last;
}

int engine_kv_write(LLMModel *m, int seq, int layer, int pos0, int npos, const float *k, const float *v,
                    char *err, size_t cap)
{
    if (m == NULL || m->dev == NULL || k == NULL || v == NULL || npos < 0) {
        seterr(err, cap, "Invalid arguments.");
        return 0;
    }
    const Config *c = &m->config;
    if (layer < 0 || layer >= c->n_layers || pos0 < 0 || pos0 > c->seq_len - npos) {
        seterr(err, cap, "KV write outside the cache (layer or positions).");
        return 0;
    }
    if (seq >= 0 && (m->batch == NULL || seq >= m->batch_seqs)) {
        seterr(err, cap, "No such batched sequence.");
        return 0;
    }
    if (seq >= 0 && pos0 > m->filled[seq]) {
        seterr(err, cap, "KV write would leave a gap after the sequence's filled positions.");
        return 0;
    }
    if (seq < -1) {
        seterr(err, cap, "Invalid sequence.");
        return 0;
    }
    if (npos == 0) return 1;
    /* the caller's rows hold every KV head; a tensor-parallel rank keeps its own */
    const size_t hs = (size_t)(c->dim / c->n_heads), kvd = hs * (size_t)c->n_kv_heads;
    const size_t c0 = (size_t)m->kv_head0 * hs, cn = (size_t)m->kv_heads * hs;
    const float *kp = k, *vp = v;
    float *tk = NULL, *tv = NULL;
    if (cn != kvd) {
        tk = (float *)malloc((size_t)npos * cn * sizeof(float));
        tv = (float *)malloc((size_t)npos * cn * sizeof(float));
        if (tk == NULL || tv == NULL) {
            free(tk);
            free(tv);
            seterr(err, cap, "Out of memory.");
            return 0;
        }
        for (int i = 0; i < npos; i++) {
            memcpy(tk + (size_t)i * cn, k + (size_t)i * kvd + c0, cn * sizeof(float));
            memcpy(tv + (size_t)i * cn, v + (size_t)i * kvd + c0, cn * sizeof(float));
        }
        kp = tk;
        vp = tv;
    }
    const int ok = seq < 0 ? pkd_kv_write(m->dev, layer, pos0, npos, kp, vp, err, cap)
                           : pkb_kv_write(m->batch, seq, layer, pos0, npos, kp, vp, err, cap);
    free(tk);
    free(tv);
    if (ok && seq >= 0 && pos0 + npos > m->filled[seq]) m->filled[seq] = pos0 + npos;
    if (ok && err && cap) err[0] = '\0';
    return ok;
}

int engine_trace(LLMModel *m, unsigned long long *out, int cap)
{
    return m == NULL ? 0 : pkd_trace(m->dev, out, cap);
}

const char *engine_last_error(const LLMModel *m)
{
    return m == NULL ? "" : m->last_error;
}

size_t engine_weight_bytes(const LLMModel *m)
{
    return m == NULL ? 0 : (size_t)m->weight_bytes;
}

int engine_launches_per_step(const LLMModel *m)
{
    return m == NULL ? 0 : pkd_launches_per_step(m->dev);
}

const Config *engine_config(const LLMModel *m)
{
    return m == NULL ? NULL : &m->config;
}

int engine_file_context(const LLMModel *m)
{
    return m == NULL ? 0 : m->file_context;
}

LLMFormat engine_format(const LLMModel *m)
{
    return m == NULL ? (LLMFormat)0 : m->format;
}

Tokenizer *engine_tokenizer(LLMModel *m)
{
    return m == NULL ? NULL : &m->tokenizer;
}

size_t engine_kv_cache_bytes(const LLMModel *m)
{
    const Config *c = engine_config(m);
    if (c == NULL) return 0;
    const size_t kvd = (size_t)(c->dim / c->n_heads * c->n_kv_heads);
    return 2u * (size_t)c->n_layers * (size_t)c->seq_len * kvd * (m->kv_half ? 2u : sizeof(float));
}

const char *engine_description(const LLMModel *m)
{
    return m == NULL ? "" : m->description;
}

int engine_is_stop_token(const LLMModel *m, int token)
{
    if (m == NULL) return 1;
    return token == m->tokenizer.eos_id;
}
