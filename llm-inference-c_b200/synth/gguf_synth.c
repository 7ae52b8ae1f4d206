/*
 * gguf_synth.c - seeded synthetic llama GGUF models and a block quantizer.
 *
 * The benchmark and the parity tests need GGUF files with the shapes of
 * TinyLlama-1.1B, Llama-2-7B and Llama-3-8B but there are no real model files
 * (and no network), so this writes random-init models: weights ~ N(0, std)
 * from a counter-based generator, quantized with the simple per-block
 * quantizers below, norms = 1.0 in F32, and a synthetic SentencePiece
 * vocabulary that the reference's GGUF tokenizer loader accepts
 * (tokenizer.ggml.model "llama", tokens/scores/token_type arrays, BOS/EOS).
 *
 * The quantizers are written from the public GGML block layouts (the same
 * layouts the reference decodes in src/gguf_quant.c); parity never depends
 * on their quality, only on the decoders reading what they wrote.
 *
 * Everything is deterministic: a weight depends only on (seed, tensor name,
 * element index), never on thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define T_F32 0
#define T_F16 1
#define T_Q4_0 2
#define T_Q8_0 8
#define T_Q4_K 12
#define T_Q5_K 13
#define T_Q6_K 14

/* ------------------------------------------------------------------ */
/* Random numbers                                                      */
/* ------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t pks_name_seed(uint64_t seed, const char *name)
{
    uint64_t h = 0xCBF29CE484222325ull ^ seed;
    for (const unsigned char *p = (const unsigned char *)name; *p; p++) {
        h = (h ^ *p) * 0x100000001B3ull;
    }
    return mix64(h);
}

/* n values of N(0, std) for elements [start, start+n) of stream `seed`
 * (Box-Muller on pairs, each pair from one 64-bit counter hash). */
void pks_gaussian(uint64_t seed, uint64_t start, size_t n, float std, float *out)
{
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) {
        uint64_t e = start + (uint64_t)i;
        uint64_t r = mix64(seed ^ mix64(e >> 1));
        double u1 = ((double)(r >> 40) + 1.0) / 16777217.0;      /* (0, 1] */
        double u2 = (double)((r >> 16) & 0xFFFFFF) / 16777216.0; /* [0, 1) */
        double rad = sqrt(-2.0 * log(u1));
        double ang = 6.283185307179586 * u2;
        double z = (e & 1) ? rad * sin(ang) : rad * cos(ang);
        out[i] = (float)(z * (double)std);
    }
}

/* Uniform integers in [lo, hi) for prompts and test inputs. */
void pks_uniform_ints(uint64_t seed, size_t n, int lo, int hi, int *out)
{
    for (size_t i = 0; i < n; i++) {
        out[i] = lo + (int)(mix64(seed ^ mix64((uint64_t)i)) % (uint64_t)(hi - lo));
    }
}

/* ------------------------------------------------------------------ */
/* Half precision (round to nearest even)                              */
/* ------------------------------------------------------------------ */

static uint16_t f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477FF000u) { /* rounds to >= 65520: overflow to inf */
        return (uint16_t)(sign | 0x7C00u);
    }
    if (ax < 0x38800000u) { /* subnormal half or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e; /* 14..24 */
        uint32_t hm = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static float h2f(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u, b;
    if (e == 31u) b = sign | 0x7F800000u | (m << 13);
    else if (e) b = sign | ((e + 112u) << 23) | (m << 13);
    else if (!m) b = sign;
    else {
        int ee = 113;
        while (!(m & 1024u)) { m <<= 1; ee--; }
        b = sign | ((uint32_t)ee << 23) | ((m & 1023u) << 13);
    }
    float f;
    memcpy(&f, &b, 4);
    return f;
}

static void put16(uint8_t *p, uint16_t v)
{
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
}

static int clampi(int v, int lo, int hi)
{
    return v < lo ? lo : (v > hi ? hi : v);
}

/* ------------------------------------------------------------------ */
/* Block quantizers                                                    */
/* ------------------------------------------------------------------ */

static void q8_0(const float *x, uint8_t *b)
{
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
    uint16_t dh = f2h(amax / 127.0f);
    float d = h2f(dh), id = d != 0.0f ? 1.0f / d : 0.0f;
    put16(b, dh);
    for (int i = 0; i < 32; i++) b[2 + i] = (uint8_t)(int8_t)clampi((int)lrintf(x[i] * id), -127, 127);
}

static void q4_0(const float *x, uint8_t *b)
{
    float vmax = 0.0f, amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); vmax = x[i]; }
    }
    uint16_t dh = f2h(vmax / -8.0f);
    float d = h2f(dh), id = d != 0.0f ? 1.0f / d : 0.0f;
    put16(b, dh);
    for (int j = 0; j < 16; j++) {
        int lo = clampi((int)lrintf(x[j] * id) + 8, 0, 15);
        int hi = clampi((int)lrintf(x[j + 16] * id) + 8, 0, 15);
        b[2 + j] = (uint8_t)(lo | (hi << 4));
    }
}

/* Shared by Q4_K (levels 15) and Q5_K (levels 31): per 32-weight sub-block
 * an affine (scale, min); 6-bit scales against fp16 super-scales d, dmin.
 * Writes header (d, dmin, scales[12]) and returns the 256 quants in q. */
static void kquant_affine(const float *x, int levels, uint8_t *hdr, int *q)
{
    float sc[8], mn[8], smax = 0.0f, mmax = 0.0f;
    for (int s = 0; s < 8; s++) {
        float lo = x[32 * s], hi = x[32 * s];
        for (int i = 1; i < 32; i++) {
            lo = fminf(lo, x[32 * s + i]);
            hi = fmaxf(hi, x[32 * s + i]);
        }
        if (lo > 0.0f) lo = 0.0f;
        sc[s] = (hi - lo) / (float)levels;
        mn[s] = -lo;
        smax = fmaxf(smax, sc[s]);
        mmax = fmaxf(mmax, mn[s]);
    }
    uint16_t dh = f2h(smax / 63.0f), mh = f2h(mmax / 63.0f);
    float d = h2f(dh), dm = h2f(mh);
    int is[8], im[8];
    for (int s = 0; s < 8; s++) {
        is[s] = d > 0.0f ? clampi((int)lrintf(sc[s] / d), 0, 63) : 0;
        im[s] = dm > 0.0f ? clampi((int)lrintf(mn[s] / dm), 0, 63) : 0;
    }
    put16(hdr, dh);
    put16(hdr + 2, mh);
    uint8_t *p = hdr + 4;
    for (int i = 0; i < 4; i++) {
        p[i] = (uint8_t)((is[i] & 63) | ((is[i + 4] >> 4) << 6));
        p[i + 4] = (uint8_t)((im[i] & 63) | ((im[i + 4] >> 4) << 6));
        p[i + 8] = (uint8_t)((is[i + 4] & 15) | ((im[i + 4] & 15) << 4));
    }
    for (int s = 0; s < 8; s++) {
        float dl = d * (float)is[s], ml = dm * (float)im[s];
        for (int i = 0; i < 32; i++) {
            q[32 * s + i] = dl > 0.0f ? clampi((int)lrintf((x[32 * s + i] + ml) / dl), 0, levels) : 0;
        }
    }
}

static void q4_k(const float *x, uint8_t *b)
{
    int q[256];
    kquant_affine(x, 15, b, q);
    for (int j = 0; j < 4; j++) {
        for (int l = 0; l < 32; l++) {
            b[16 + 32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
        }
    }
}

static void q5_k(const float *x, uint8_t *b)
{
    int q[256];
    kquant_affine(x, 31, b, q);
    uint8_t *qh = b + 16, *qs = b + 48;
    memset(qh, 0, 32);
    for (int j = 0; j < 4; j++) {
        for (int l = 0; l < 32; l++) {
            int a = q[64 * j + l], c = q[64 * j + 32 + l];
            qs[32 * j + l] = (uint8_t)((a & 15) | ((c & 15) << 4));
            qh[l] |= (uint8_t)(((a >> 4) & 1) << (2 * j));
            qh[l] |= (uint8_t)(((c >> 4) & 1) << (2 * j + 1));
        }
    }
}

static void q6_k(const float *x, uint8_t *b)
{
    float gs[16], amax = 0.0f;
    for (int g = 0; g < 16; g++) {
        float v = 0.0f, av = 0.0f;
        for (int i = 0; i < 16; i++) {
            if (fabsf(x[16 * g + i]) > av) { av = fabsf(x[16 * g + i]); v = x[16 * g + i]; }
        }
        gs[g] = v / -32.0f;
        amax = fmaxf(amax, fabsf(gs[g]));
    }
    uint16_t dh = f2h(amax / 127.0f);
    float d = h2f(dh);
    int8_t sc[16];
    int q[256];
    for (int g = 0; g < 16; g++) {
        sc[g] = (int8_t)(d > 0.0f ? clampi((int)lrintf(gs[g] / d), -127, 127) : 0);
        float s = d * (float)sc[g];
        for (int i = 0; i < 16; i++) {
            q[16 * g + i] = (s != 0.0f ? clampi((int)lrintf(x[16 * g + i] / s), -32, 31) : 0) + 32;
        }
    }
    uint8_t *ql = b, *qh = b + 128;
    for (int h = 0; h < 2; h++) {
        for (int l = 0; l < 32; l++) {
            const int *qq = q + 128 * h;
            ql[64 * h + l] = (uint8_t)((qq[l] & 15) | ((qq[64 + l] & 15) << 4));
            ql[64 * h + 32 + l] = (uint8_t)((qq[32 + l] & 15) | ((qq[96 + l] & 15) << 4));
            qh[32 * h + l] = (uint8_t)((qq[l] >> 4) | ((qq[32 + l] >> 4) << 2) |
                                       ((qq[64 + l] >> 4) << 4) | ((qq[96 + l] >> 4) << 6));
        }
    }
    memcpy(b + 192, sc, 16);
    put16(b + 208, dh);
}

/* Bytes for n weights of `type`, or 0 if n is not a whole number of blocks. */
uint64_t pks_type_bytes(uint32_t type, uint64_t n)
{
    switch (type) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q4_0: return n % 32 ? 0 : n / 32 * 18;
    case T_Q8_0: return n % 32 ? 0 : n / 32 * 34;
    case T_Q4_K: return n % 256 ? 0 : n / 256 * 144;
    case T_Q5_K: return n % 256 ? 0 : n / 256 * 176;
    case T_Q6_K: return n % 256 ? 0 : n / 256 * 210;
    default: return 0;
    }
}

/* Quantize n weights (a whole number of blocks) to `type`. Returns 1 on
 * success, 0 for an unsupported type or a partial block. */
int pks_quantize(uint32_t type, const float *x, uint64_t n, void *out)
{
    uint8_t *o = (uint8_t *)out;
    if (pks_type_bytes(type, n) == 0 && n != 0) return 0;
    switch (type) {
    case T_F32: memcpy(o, x, n * 4); return 1;
    case T_F16:
        for (uint64_t i = 0; i < n; i++) put16(o + 2 * i, f2h(x[i]));
        return 1;
    default: break;
    }
    long long nb = (long long)(type == T_Q4_0 || type == T_Q8_0 ? n / 32 : n / 256);
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < nb; i++) {
        switch (type) {
        case T_Q4_0: q4_0(x + 32 * i, o + 18 * i); break;
        case T_Q8_0: q8_0(x + 32 * i, o + 34 * i); break;
        case T_Q4_K: q4_k(x + 256 * i, o + 144 * i); break;
        case T_Q5_K: q5_k(x + 256 * i, o + 176 * i); break;
        case T_Q6_K: q6_k(x + 256 * i, o + 210 * i); break;
        }
    }
    return 1;
}

/* ------------------------------------------------------------------ */
/* GGUF writer                                                         */
/* ------------------------------------------------------------------ */

/* Model description. Types are GGML type ids. */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, context_length;
    float rope_theta, rms_eps, weight_std;
    uint64_t seed;
    uint32_t t_embd, t_output, t_q, t_k, t_v_even, t_v_odd, t_o, t_gate, t_up, t_down_even,
        t_down_odd;
    int tied_output; /* 1: omit output.weight (output tied to token_embd) */
    int space_piece; /* 1: token 259 is the bare word-start piece, so that a
                        SentencePiece encoder can tokenize any text (space + bytes) */
} PksSpec;

typedef struct {
    char name[64];
    uint32_t type, ndim;
    uint64_t dims[2], offset, bytes;
    int norm;
} WT;

static void w_u32(FILE *f, uint32_t v) { fwrite(&v, 4, 1, f); }
static void w_u64(FILE *f, uint64_t v) { fwrite(&v, 8, 1, f); }
static void w_str(FILE *f, const char *s)
{
    w_u64(f, strlen(s));
    fwrite(s, 1, strlen(s), f);
}
static void kv_u32(FILE *f, const char *k, uint32_t v) { w_str(f, k); w_u32(f, 4); w_u32(f, v); }
static void kv_f32(FILE *f, const char *k, float v)
{
    w_str(f, k);
    w_u32(f, 6);
    fwrite(&v, 4, 1, f);
}
static void kv_str(FILE *f, const char *k, const char *v) { w_str(f, k); w_u32(f, 8); w_str(f, v); }

static void token_text(int i, int space_piece, char *buf, size_t cap)
{
    if (i == 0) snprintf(buf, cap, "<unk>");
    else if (i == 1) snprintf(buf, cap, "<s>");
    else if (i == 2) snprintf(buf, cap, "</s>");
    else if (i < 259) snprintf(buf, cap, "<0x%02X>", i - 3);
    else if (i == 259 && space_piece) snprintf(buf, cap, "\xE2\x96\x81"); /* "▁" */
    else snprintf(buf, cap, "\xE2\x96\x81t%d", i); /* "▁t<i>": unique normal pieces */
}

static int token_type(int i)
{
    if (i == 0) return 2;      /* unknown */
    if (i < 3) return 3;       /* control */
    if (i < 259) return 6;     /* byte */
    return 1;                  /* normal */
}

static int add_t(WT *t, int *n, const char *name, uint32_t type, uint64_t cols, uint64_t rows,
                 int norm)
{
    WT *w = &t[(*n)++];
    snprintf(w->name, sizeof(w->name), "%s", name);
    w->type = type;
    w->ndim = rows ? 2 : 1;
    w->dims[0] = cols;
    w->dims[1] = rows;
    w->bytes = pks_type_bytes(type, cols * (rows ? rows : 1));
    w->norm = norm;
    return w->bytes != 0;
}

/* Write a synthetic llama GGUF v3 file. Returns 1 on success. */
int pks_write_model(const char *path, const PksSpec *s, char *err, size_t cap)
{
    if (path == NULL || s == NULL || s->dim <= 0 || s->n_layers <= 0 || s->n_heads <= 0 ||
        s->n_kv_heads <= 0 || s->vocab_size < 260 || s->dim % s->n_heads) {
        if (err && cap) snprintf(err, cap, "invalid spec");
        return 0;
    }
    const uint64_t dim = (uint64_t)s->dim, hid = (uint64_t)s->hidden_dim;
    const uint64_t kvd = dim / (uint64_t)s->n_heads * (uint64_t)s->n_kv_heads;
    const int nmax = 3 + 9 * s->n_layers;
    WT *t = (WT *)calloc((size_t)nmax, sizeof(WT));
    int n = 0, ok = 1;
    char nm[64];
    ok &= add_t(t, &n, "token_embd.weight", s->t_embd, dim, (uint64_t)s->vocab_size, 0);
    for (int l = 0; l < s->n_layers; l++) {
#define L(suffix, type, cols, rows, norm) \
    (snprintf(nm, sizeof(nm), "blk.%d.%s", l, suffix), add_t(t, &n, nm, type, cols, rows, norm))
        ok &= L("attn_norm.weight", T_F32, dim, 0, 1);
        ok &= L("attn_q.weight", s->t_q, dim, dim, 0);
        ok &= L("attn_k.weight", s->t_k, dim, kvd, 0);
        ok &= L("attn_v.weight", (l % 2 == 0) ? s->t_v_even : s->t_v_odd, dim, kvd, 0);
        ok &= L("attn_output.weight", s->t_o, dim, dim, 0);
        ok &= L("ffn_norm.weight", T_F32, dim, 0, 1);
        ok &= L("ffn_gate.weight", s->t_gate, dim, hid, 0);
        ok &= L("ffn_up.weight", s->t_up, dim, hid, 0);
        ok &= L("ffn_down.weight", (l % 2 == 0) ? s->t_down_even : s->t_down_odd, hid, dim, 0);
#undef L
    }
    ok &= add_t(t, &n, "output_norm.weight", T_F32, dim, 0, 1);
    if (!s->tied_output) ok &= add_t(t, &n, "output.weight", s->t_output, dim, (uint64_t)s->vocab_size, 0);
    if (!ok) {
        free(t);
        if (err && cap) snprintf(err, cap, "a shape is not a whole number of blocks");
        return 0;
    }
    uint64_t off = 0;
    for (int i = 0; i < n; i++) {
        t[i].offset = off;
        off += (t[i].bytes + 31) / 32 * 32;
    }

    FILE *f = fopen(path, "wb");
    if (f == NULL) {
        free(t);
        if (err && cap) snprintf(err, cap, "cannot create %s", path);
        return 0;
    }
    fwrite("GGUF", 1, 4, f);
    w_u32(f, 3);
    w_u64(f, (uint64_t)n);
    w_u64(f, 18);
    kv_str(f, "general.architecture", "llama");
    kv_str(f, "general.name", "synthetic");
    kv_u32(f, "llama.context_length", (uint32_t)s->context_length);
    kv_u32(f, "llama.embedding_length", (uint32_t)s->dim);
    kv_u32(f, "llama.block_count", (uint32_t)s->n_layers);
    kv_u32(f, "llama.feed_forward_length", (uint32_t)s->hidden_dim);
    kv_u32(f, "llama.attention.head_count", (uint32_t)s->n_heads);
    kv_u32(f, "llama.attention.head_count_kv", (uint32_t)s->n_kv_heads);
    kv_u32(f, "llama.rope.dimension_count", (uint32_t)(s->dim / s->n_heads));
    kv_f32(f, "llama.rope.freq_base", s->rope_theta);
    kv_f32(f, "llama.attention.layer_norm_rms_epsilon", s->rms_eps);
    kv_str(f, "tokenizer.ggml.model", "llama");
    {
        char buf[32];
        w_str(f, "tokenizer.ggml.tokens");
        w_u32(f, 9);
        w_u32(f, 8);
        w_u64(f, (uint64_t)s->vocab_size);
        for (int i = 0; i < s->vocab_size; i++) {
            token_text(i, s->space_piece, buf, sizeof(buf));
            w_str(f, buf);
        }
        w_str(f, "tokenizer.ggml.scores");
        w_u32(f, 9);
        w_u32(f, 6);
        w_u64(f, (uint64_t)s->vocab_size);
        for (int i = 0; i < s->vocab_size; i++) {
            float sc = token_type(i) == 1 ? -(float)i : 0.0f;
            fwrite(&sc, 4, 1, f);
        }
        w_str(f, "tokenizer.ggml.token_type");
        w_u32(f, 9);
        w_u32(f, 5);
        w_u64(f, (uint64_t)s->vocab_size);
        for (int i = 0; i < s->vocab_size; i++) {
            int32_t ty = token_type(i);
            fwrite(&ty, 4, 1, f);
        }
    }
    kv_u32(f, "tokenizer.ggml.bos_token_id", 1);
    kv_u32(f, "tokenizer.ggml.eos_token_id", 2);
    kv_u32(f, "general.alignment", 32);
    for (int i = 0; i < n; i++) {
        w_str(f, t[i].name);
        w_u32(f, t[i].ndim);
        for (uint32_t d = 0; d < t[i].ndim; d++) w_u64(f, t[i].dims[d]);
        w_u32(f, t[i].type);
        w_u64(f, t[i].offset);
    }
    long pos = ftell(f);
    static const uint8_t zeros[64] = {0};
    fwrite(zeros, 1, (size_t)((32 - pos % 32) % 32), f);

    /* Tensor data, generated and quantized a chunk of rows at a time. */
    const uint64_t chunk_w = 1u << 22;
    float *buf = (float *)malloc(chunk_w * 4);
    uint8_t *qb = (uint8_t *)malloc(chunk_w * 4);
    for (int i = 0; i < n && ok; i++) {
        const uint64_t cols = t[i].dims[0], rows = t[i].ndim == 2 ? t[i].dims[1] : 1;
        const uint64_t seed = pks_name_seed(s->seed, t[i].name);
        uint64_t rows_per = chunk_w / cols;
        if (rows_per == 0) rows_per = 1;
        for (uint64_t r = 0; r < rows && ok; r += rows_per) {
            uint64_t nr = rows - r < rows_per ? rows - r : rows_per;
            uint64_t cnt = nr * cols;
            if (t[i].norm) {
                for (uint64_t k = 0; k < cnt; k++) buf[k] = 1.0f;
            } else {
                pks_gaussian(seed, r * cols, (size_t)cnt, s->weight_std, buf);
            }
            ok &= pks_quantize(t[i].type, buf, cnt, qb);
            uint64_t nbytes = pks_type_bytes(t[i].type, cnt);
            ok &= fwrite(qb, 1, nbytes, f) == nbytes;
        }
        uint64_t pad = (32 - t[i].bytes % 32) % 32;
        fwrite(zeros, 1, (size_t)pad, f);
    }
    free(buf);
    free(qb);
    ok &= fclose(f) == 0;
    free(t);
    if (!ok && err && cap) snprintf(err, cap, "write failed");
    return ok;
}
