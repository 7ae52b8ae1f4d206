/*
 * oracle.c - CPU restatement of the GGUF quantized decode path of
 * Gopichand1401/llm-inference-c (pocketllm), used ONLY as test
 * infrastructure: the parity tests, smoke() and the bench's CPU-baseline leg
 * call it as the checker. Nothing in the product links or loads it.
 *
 * Every function restates the reference's arithmetic in the same order so
 * that, compiled with the reference's flags (gcc -std=c11 -O2, which implies
 * -ffp-contract=off: no fused multiply-add), results are bit-identical to the
 * reference. That claim is pinned by tests/test_oracle_pins.py against the
 * reference itself (built from its own sources into oracle/_ref) and against
 * gguf-py golden vectors committed under tests/golden/.
 *
 * Citations are path:line inside the reference project.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORC_F32 0
#define ORC_F16 1
#define ORC_Q4_0 2
#define ORC_Q8_0 8
#define ORC_Q4_K 12
#define ORC_Q5_K 13
#define ORC_Q6_K 14

/* ------------------------------------------------------------------ */
/* Scalar helpers                                                      */
/* ------------------------------------------------------------------ */

/* IEEE half -> float, subnormals normalised, inf/NaN keep their payload.
 * Follows src/gguf_quant.c:6-59. */
float orc_fp16_to_fp32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 31u;
    uint32_t man = h & 1023u;
    uint32_t bits;

    if (exp == 31u) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp != 0u) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0u) {
        bits = sign;
    } else {
        /* Subnormal: shift the leading one up to bit 10. */
        int e = 113;
        while (!(man & 1024u)) {
            man <<= 1;
            e--;
        }
        bits = sign | ((uint32_t)e << 23) | ((man & 1023u) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t rd16(const uint8_t *p)
{
    return (uint16_t)(p[0] | (p[1] << 8));
}

/* 6-bit (scale, min) pair `i` of the 12 packed bytes, src/gguf_quant.c:65-90. */
int orc_q4k_scale_min(const uint8_t *s, unsigned i, uint8_t *sc, uint8_t *mn)
{
    if (s == NULL || sc == NULL || mn == NULL || i >= 8) {
        return 0;
    }
    if (i < 4) {
        *sc = s[i] & 63;
        *mn = s[i + 4] & 63;
    } else {
        *sc = (uint8_t)((s[i + 4] & 15) | ((s[i - 4] >> 6) << 4));
        *mn = (uint8_t)((s[i + 4] >> 4) | ((s[i] >> 6) << 4));
    }
    return 1;
}

/* Block geometry, src/gguf_quant.c:351-368. */
int orc_block_info(uint32_t type, size_t *weights, size_t *bytes)
{
    size_t w, b;
    switch (type) {
    case ORC_Q4_0: w = 32; b = 18; break;
    case ORC_Q8_0: w = 32; b = 34; break;
    case ORC_Q4_K: w = 256; b = 144; break;
    case ORC_Q5_K: w = 256; b = 176; break;
    case ORC_Q6_K: w = 256; b = 210; break;
    default: return 0;
    }
    if (weights) *weights = w;
    if (bytes) *bytes = b;
    return 1;
}

/* ------------------------------------------------------------------ */
/* Block decoders (bit-exact), src/gguf_quant.c:92-345                 */
/* ------------------------------------------------------------------ */

/* Q4_K: w = (d*sc)*q - (dmin*m), src/gguf_quant.c:92-161. */
static void dec_q4k(const uint8_t *b, float *o)
{
    const float d = orc_fp16_to_fp32(rd16(b));
    const float dmin = orc_fp16_to_fp32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qs = b + 16;
    for (int j = 0; j < 4; j++) {
        uint8_t s0, m0, s1, m1;
        orc_q4k_scale_min(sc, 2 * j, &s0, &m0);
        orc_q4k_scale_min(sc, 2 * j + 1, &s1, &m1);
        const float dl = d * (float)s0, ml = dmin * (float)m0;
        const float dh = d * (float)s1, mh = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            o[64 * j + l] = dl * (float)(qs[32 * j + l] & 15) - ml;
            o[64 * j + 32 + l] = dh * (float)(qs[32 * j + l] >> 4) - mh;
        }
    }
}

/* Q5_K: Q4_K plus bit 2j / 2j+1 of qh[l], src/gguf_quant.c:307-345. */
static void dec_q5k(const uint8_t *b, float *o)
{
    const float d = orc_fp16_to_fp32(rd16(b));
    const float dmin = orc_fp16_to_fp32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qh = b + 16, *qs = b + 48;
    for (int j = 0; j < 4; j++) {
        uint8_t s0, m0, s1, m1;
        orc_q4k_scale_min(sc, 2 * j, &s0, &m0);
        orc_q4k_scale_min(sc, 2 * j + 1, &s1, &m1);
        const float dl = d * (float)s0, ml = dmin * (float)m0;
        const float dh = d * (float)s1, mh = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            unsigned ql = (qs[32 * j + l] & 15u) + (((qh[l] >> (2 * j)) & 1u) << 4);
            unsigned qhi = (qs[32 * j + l] >> 4) + (((qh[l] >> (2 * j + 1)) & 1u) << 4);
            o[64 * j + l] = dl * (float)ql - ml;
            o[64 * j + 32 + l] = dh * (float)qhi - mh;
        }
    }
}

/* Q6_K 6-bit unpack in output order, src/gguf_quant.c:185-217. */
static void unpack_q6k(const uint8_t *b, int8_t *q)
{
    for (int h = 0; h < 2; h++) {
        const uint8_t *ql = b + 64 * h, *qh = b + 128 + 32 * h;
        for (int l = 0; l < 32; l++) {
            unsigned hb = qh[l];
            q[128 * h + l] = (int8_t)((int)((ql[l] & 15u) | ((hb & 3u) << 4)) - 32);
            q[128 * h + 32 + l] = (int8_t)((int)((ql[l + 32] & 15u) | (((hb >> 2) & 3u) << 4)) - 32);
            q[128 * h + 64 + l] = (int8_t)((int)((ql[l] >> 4) | (((hb >> 4) & 3u) << 4)) - 32);
            q[128 * h + 96 + l] = (int8_t)((int)((ql[l + 32] >> 4) | (((hb >> 6) & 3u) << 4)) - 32);
        }
    }
}

/* Q6_K: w = (d*sc[i/16])*q, src/gguf_quant.c:219-252. */
static void dec_q6k(const uint8_t *b, float *o)
{
    int8_t q[256];
    unpack_q6k(b, q);
    const float d = orc_fp16_to_fp32(rd16(b + 208));
    const int8_t *sc = (const int8_t *)(b + 192);
    for (int g = 0; g < 16; g++) {
        const float gs = d * (float)sc[g];
        for (int k = 0; k < 16; k++) {
            o[16 * g + k] = gs * (float)q[16 * g + k];
        }
    }
}

/* Q4_0: w = d*(q-8), low nibbles first, src/gguf_quant.c:258-275. */
static void dec_q4_0(const uint8_t *b, float *o)
{
    const float d = orc_fp16_to_fp32(rd16(b));
    for (int j = 0; j < 16; j++) {
        o[j] = d * (float)((int)(b[2 + j] & 15) - 8);
        o[j + 16] = d * (float)((int)(b[2 + j] >> 4) - 8);
    }
}

/* Q8_0: w = q*d, src/gguf_quant.c:281-295. */
static void dec_q8_0(const uint8_t *b, float *o)
{
    const float d = orc_fp16_to_fp32(rd16(b));
    for (int j = 0; j < 32; j++) {
        o[j] = (float)(int8_t)b[2 + j] * d;
    }
}

/* Type dispatch, src/gguf_quant.c:371-407. */
int orc_dequantize_block(uint32_t type, const void *src, float *out)
{
    const uint8_t *b = (const uint8_t *)src;
    if (b == NULL || out == NULL) return 0;
    switch (type) {
    case ORC_Q4_0: dec_q4_0(b, out); return 1;
    case ORC_Q8_0: dec_q8_0(b, out); return 1;
    case ORC_Q4_K: dec_q4k(b, out); return 1;
    case ORC_Q5_K: dec_q5k(b, out); return 1;
    case ORC_Q6_K: dec_q6k(b, out); return 1;
    default: return 0;
    }
}

/* Decode `nblocks` consecutive blocks (test convenience). */
int orc_dequantize_blocks(uint32_t type, const void *src, size_t nblocks, float *out)
{
    size_t bw, bb;
    if (!orc_block_info(type, &bw, &bb)) return 0;
    for (size_t i = 0; i < nblocks; i++) {
        if (!orc_dequantize_block(type, (const uint8_t *)src + i * bb, out + i * bw)) return 0;
    }
    return 1;
}

/* Row bytes for `cols` columns of `type`; 0 if not a whole number of blocks. */
uint64_t orc_row_bytes(uint32_t type, uint64_t cols)
{
    size_t bw, bb;
    if (type == ORC_F32) return cols * 4;
    if (type == ORC_F16) return cols * 2;
    if (!orc_block_info(type, &bw, &bb) || cols % bw) return 0;
    return cols / bw * bb;
}

/* One row to FP32, src/gguf_model.c:314-359. */
int orc_dequantize_row(uint32_t type, const void *row, uint64_t cols, float *out)
{
    const uint8_t *p = (const uint8_t *)row;
    if (p == NULL || out == NULL) return 0;
    if (type == ORC_F32) {
        memcpy(out, p, cols * 4);
        return 1;
    }
    if (type == ORC_F16) {
        for (uint64_t i = 0; i < cols; i++) out[i] = orc_fp16_to_fp32(rd16(p + 2 * i));
        return 1;
    }
    size_t bw, bb;
    if (!orc_block_info(type, &bw, &bb)) return 0;
    for (uint64_t b = 0; b < cols / bw; b++) {
        orc_dequantize_block(type, p + b * bb, out + b * bw);
    }
    return 1;
}

/* ------------------------------------------------------------------ */
/* Matrix-vector products, src/gguf_model.c:363-771                   */
/* ------------------------------------------------------------------ */

/* Decode-then-dot in column order, src/gguf_model.c:371-414. */
static float dot_in_column_order(uint32_t type, const uint8_t *row, uint64_t cols, const float *x)
{
    float acc = 0.0f;
    if (type == ORC_F32) {
        for (uint64_t i = 0; i < cols; i++) {
            float v;
            memcpy(&v, row + 4 * i, 4);
            acc += v * x[i];
        }
        return acc;
    }
    if (type == ORC_F16) {
        for (uint64_t i = 0; i < cols; i++) acc += orc_fp16_to_fp32(rd16(row + 2 * i)) * x[i];
        return acc;
    }
    float w[256];
    size_t bw, bb;
    orc_block_info(type, &bw, &bb);
    for (uint64_t b = 0; b < cols / bw; b++) {
        orc_dequantize_block(type, row + b * bb, w);
        for (size_t i = 0; i < bw; i++) acc += w[i] * x[b * bw + i];
    }
    return acc;
}

static int type_ok(uint32_t type)
{
    return type == ORC_F32 || type == ORC_F16 || orc_block_info(type, NULL, NULL);
}

/* gguf_matvec_reference, src/gguf_model.c:416-439. */
int orc_matvec_reference(uint32_t type, const void *data, uint64_t rows, uint64_t cols,
                         const float *x, float *y)
{
    uint64_t rb = orc_row_bytes(type, cols);
    if (data == NULL || x == NULL || y == NULL || !type_ok(type) || rb == 0) return 0;
    #pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)rows; r++) {
        y[r] = dot_in_column_order(type, (const uint8_t *)data + (size_t)r * rb, cols, x);
    }
    return 1;
}

/* Fixed pairwise tree over 32 values: v[l] += v[l+w] for w = 16,8,4,2,1. */
static inline float tree32(float *v)
{
    for (int w = 16; w > 0; w >>= 1) {
        for (int l = 0; l < w; l++) v[l] += v[l + w];
    }
    return v[0];
}

/* q4k_row_dot_fast, src/gguf_model.c:457-507. */
static float dot_q4k(const uint8_t *row, const float *x, const float *xs32, size_t nb)
{
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * 144;
        const float d = orc_fp16_to_fp32(rd16(blk));
        const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
        for (int j = 0; j < 4; j++) {
            uint8_t s0, m0, s1, m1;
            orc_q4k_scale_min(blk + 4, 2 * j, &s0, &m0);
            orc_q4k_scale_min(blk + 4, 2 * j + 1, &s1, &m1);
            const uint8_t *q = blk + 16 + 32 * j;
            const float *xa = x + 256 * b + 64 * j;
            float lo[32], hi[32];
            for (int l = 0; l < 32; l++) {
                lo[l] = (float)(q[l] & 15) * xa[l];
                hi[l] = (float)(q[l] >> 4) * xa[32 + l];
            }
            const float slo = tree32(lo), shi = tree32(hi);
            total += d * (float)s0 * slo - dmin * (float)m0 * xs32[8 * b + 2 * j];
            total += d * (float)s1 * shi - dmin * (float)m1 * xs32[8 * b + 2 * j + 1];
        }
    }
    return total;
}

/* q5k_row_dot_fast, src/gguf_model.c:574-626. */
static float dot_q5k(const uint8_t *row, const float *x, const float *xs32, size_t nb)
{
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * 176;
        const float d = orc_fp16_to_fp32(rd16(blk));
        const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
        const uint8_t *qh = blk + 16, *qs = blk + 48;
        for (int j = 0; j < 4; j++) {
            uint8_t s0, m0, s1, m1;
            orc_q4k_scale_min(blk + 4, 2 * j, &s0, &m0);
            orc_q4k_scale_min(blk + 4, 2 * j + 1, &s1, &m1);
            const uint8_t *q = qs + 32 * j;
            const float *xa = x + 256 * b + 64 * j;
            float lo[32], hi[32];
            for (int l = 0; l < 32; l++) {
                unsigned a = (q[l] & 15u) | (((qh[l] >> (2 * j)) & 1u) << 4);
                unsigned c = (q[l] >> 4) | (((qh[l] >> (2 * j + 1)) & 1u) << 4);
                lo[l] = (float)a * xa[l];
                hi[l] = (float)c * xa[32 + l];
            }
            const float slo = tree32(lo), shi = tree32(hi);
            total += d * (float)s0 * slo - dmin * (float)m0 * xs32[8 * b + 2 * j];
            total += d * (float)s1 * shi - dmin * (float)m1 * xs32[8 * b + 2 * j + 1];
        }
    }
    return total;
}

/* q6k_row_dot_fast, src/gguf_model.c:516-566. */
static float dot_q6k(const uint8_t *row, const float *x, size_t nb)
{
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * 210;
        int8_t q[256];
        unpack_q6k(blk, q);
        const float d = orc_fp16_to_fp32(rd16(blk + 208));
        const int8_t *sc = (const int8_t *)(blk + 192);
        const float *xb = x + 256 * b;
        for (int g = 0; g < 16; g++) {
            const int8_t *qg = q + 16 * g;
            const float *xg = xb + 16 * g;
            float a[8];
            for (int k = 0; k < 8; k++) {
                a[k] = (float)qg[k] * xg[k] + (float)qg[k + 8] * xg[k + 8];
            }
            const float s = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
            total += d * (float)sc[g] * s;
        }
    }
    return total;
}

/* q4_0_row_dot_fast, src/gguf_model.c:633-661. */
static float dot_q4_0(const uint8_t *row, const float *x, size_t nb)
{
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * 18;
        const float *xb = x + 32 * b;
        float t[32];
        for (int l = 0; l < 16; l++) {
            t[l] = (float)((int)(blk[2 + l] & 15) - 8) * xb[l];
            t[l + 16] = (float)((int)(blk[2 + l] >> 4) - 8) * xb[l + 16];
        }
        total += orc_fp16_to_fp32(rd16(blk)) * tree32(t);
    }
    return total;
}

/* q8_0_row_dot_fast, src/gguf_model.c:664-691. */
static float dot_q8_0(const uint8_t *row, const float *x, size_t nb)
{
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * 34;
        const float *xb = x + 32 * b;
        float t[32];
        for (int l = 0; l < 32; l++) t[l] = (float)(int8_t)blk[2 + l] * xb[l];
        total += orc_fp16_to_fp32(rd16(blk)) * tree32(t);
    }
    return total;
}

/* Sums of x over 32-input groups, src/gguf_model.c:743-753. */
void orc_xsum32(const float *x, size_t groups, float *xs)
{
    for (size_t g = 0; g < groups; g++) {
        float s = 0.0f;
        for (int i = 0; i < 32; i++) s += x[g * 32 + i];
        xs[g] = s;
    }
}

/* gguf_matvec (fast path dispatch), src/gguf_model.c:693-771. */
int orc_matvec(uint32_t type, const void *data, uint64_t rows, uint64_t cols,
               const float *x, float *y)
{
    uint64_t rb = orc_row_bytes(type, cols);
    if (data == NULL || x == NULL || y == NULL || !type_ok(type) || rb == 0) return 0;
    size_t bw;
    if (!orc_block_info(type, &bw, NULL)) {
        return orc_matvec_reference(type, data, rows, cols, x, y);
    }
    const uint8_t *base = (const uint8_t *)data;
    const size_t nb = (size_t)(cols / bw);
    float *xs = NULL;
    if (type == ORC_Q4_K || type == ORC_Q5_K) {
        xs = (float *)malloc(nb * 8 * sizeof(float));
        if (xs == NULL) return orc_matvec_reference(type, data, rows, cols, x, y);
        orc_xsum32(x, nb * 8, xs);
    }
    #pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)rows; r++) {
        const uint8_t *row = base + (size_t)r * rb;
        float v = 0.0f;
        switch (type) {
        case ORC_Q4_K: v = dot_q4k(row, x, xs, nb); break;
        case ORC_Q5_K: v = dot_q5k(row, x, xs, nb); break;
        case ORC_Q6_K: v = dot_q6k(row, x, nb); break;
        case ORC_Q4_0: v = dot_q4_0(row, x, nb); break;
        case ORC_Q8_0: v = dot_q8_0(row, x, nb); break;
        }
        y[r] = v;
    }
    free(xs);
    return 1;
}

/* ------------------------------------------------------------------ */
/* Minimal GGUF reader (config keys of src/checkpoint_gguf.c:435-758,   */
/* tensor directory :780-900, data offset :905-1030)                    */
/* ------------------------------------------------------------------ */

typedef struct {
    char name[96];
    uint32_t ndim, type;
    uint64_t dims[4], offset;
} OrcTensor;

typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
    int rope_dim;
    float rope_freq_base, rms_norm_eps, rope_scale;
} OrcConfig;

typedef struct {
    uint32_t type;
    const uint8_t *data;
    uint64_t rows, cols, row_bytes;
} OrcWeight;

typedef struct {
    OrcWeight wq, wk, wv, wo, gate, up, down;
    const float *attn_norm, *ffn_norm; /* decoded at open (src/gguf_forward.c:116-144) */
} OrcLayer;

typedef struct {
    OrcConfig c;
    int file_context;
    uint8_t *file;
    size_t file_size;
    OrcTensor *t;
    uint64_t nt;
    uint64_t data_off;
    OrcWeight embd, output;
    OrcLayer *layers;
    float *norms;
    /* RunState, src/model.c:33-100 */
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits, *kc, *vc;
    int kv_half; /* not in the reference: cache entries rounded to IEEE half */
} OrcModel;

typedef struct {
    const uint8_t *p;
    size_t n, pos;
    int bad;
} Cur;

static uint64_t cur_u(Cur *c, int bytes)
{
    if (c->bad || c->pos + (size_t)bytes > c->n) {
        c->bad = 1;
        return 0;
    }
    uint64_t v = 0;
    for (int i = 0; i < bytes; i++) v |= (uint64_t)c->p[c->pos + i] << (8 * i);
    c->pos += (size_t)bytes;
    return v;
}

static const char *cur_str(Cur *c, uint64_t *len)
{
    *len = cur_u(c, 8);
    if (c->bad || *len > c->n - c->pos) {
        c->bad = 1;
        return NULL;
    }
    const char *s = (const char *)c->p + c->pos;
    c->pos += (size_t)*len;
    return s;
}

static int scalar_size(uint32_t t)
{
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    return t < 13 ? sz[t] : -1;
}

static void cur_skip(Cur *c, uint32_t t)
{
    uint64_t len;
    if (t == 8) {
        cur_str(c, &len);
    } else if (t == 9) {
        uint32_t et = (uint32_t)cur_u(c, 4);
        uint64_t n = cur_u(c, 8);
        if (et == 9 || et > 12) {
            c->bad = 1;
            return;
        }
        for (uint64_t i = 0; i < n && !c->bad; i++) cur_skip(c, et);
    } else if (scalar_size(t) > 0) {
        c->pos += (size_t)scalar_size(t);
        if (c->pos > c->n) c->bad = 1;
    } else {
        c->bad = 1;
    }
}

static int key_eq(const char *k, uint64_t n, const char *s)
{
    return strlen(s) == n && memcmp(k, s, n) == 0;
}

static const OrcTensor *find_t(const OrcModel *m, const char *name)
{
    for (uint64_t i = 0; i < m->nt; i++) {
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    }
    return NULL;
}

/* bind_weight, src/gguf_model.c:44-128 (rows == 0 means a 1-D tensor). */
static int bind(OrcModel *m, const char *name, uint64_t cols, uint64_t rows, OrcWeight *w)
{
    const OrcTensor *t = find_t(m, name);
    if (t == NULL) return 0;
    uint32_t nd = rows == 0 ? 1 : 2;
    if (t->ndim != nd || t->dims[0] != cols || (nd == 2 && t->dims[1] != rows)) return 0;
    if (!type_ok(t->type)) return 0;
    uint64_t rb = orc_row_bytes(t->type, cols);
    uint64_t nr = rows == 0 ? 1 : rows;
    if (rb == 0 || m->data_off + t->offset + rb * nr > m->file_size) return 0;
    w->type = t->type;
    w->data = m->file + m->data_off + t->offset;
    w->rows = nr;
    w->cols = cols;
    w->row_bytes = rb;
    return 1;
}

static void seterr(char *e, size_t cap, const char *msg)
{
    if (e && cap) snprintf(e, cap, "%s", msg);
}

void orc_close(OrcModel *m);

/* Open a llama GGUF file and allocate the run state for min(file context,
 * max_context or 4096) positions (src/engine.c:143-162). */
OrcModel *orc_open(const char *path, int max_context, char *err, size_t cap)
{
    FILE *f = fopen(path, "rb");
    if (f == NULL) {
        seterr(err, cap, "cannot open");
        return NULL;
    }
    OrcModel *m = (OrcModel *)calloc(1, sizeof(*m));
    fseek(f, 0, SEEK_END);
    m->file_size = (size_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    m->file = (uint8_t *)malloc(m->file_size);
    if (m->file == NULL || fread(m->file, 1, m->file_size, f) != m->file_size) {
        fclose(f);
        seterr(err, cap, "cannot read");
        orc_close(m);
        return NULL;
    }
    fclose(f);

    Cur c = {m->file, m->file_size, 0, 0};
    if (m->file_size < 24 || memcmp(m->file, "GGUF", 4) != 0) {
        seterr(err, cap, "not gguf");
        orc_close(m);
        return NULL;
    }
    c.pos = 4;
    uint32_t ver = (uint32_t)cur_u(&c, 4);
    m->nt = cur_u(&c, 8);
    uint64_t nkv = cur_u(&c, 8);
    if (ver < 2 || ver > 3) {
        seterr(err, cap, "bad version");
        orc_close(m);
        return NULL;
    }
    OrcConfig k = {0};
    uint32_t align = 32;
    char scal_type[32] = "";
    float scal_factor = 0.0f, scal_old = 0.0f;
    for (uint64_t i = 0; i < nkv && !c.bad; i++) {
        uint64_t kl;
        const char *key = cur_str(&c, &kl);
        uint32_t t = (uint32_t)cur_u(&c, 4);
        if (c.bad) break;
        int *dst = NULL;
        if (key_eq(key, kl, "llama.embedding_length")) dst = &k.dim;
        else if (key_eq(key, kl, "llama.feed_forward_length")) dst = &k.hidden_dim;
        else if (key_eq(key, kl, "llama.block_count")) dst = &k.n_layers;
        else if (key_eq(key, kl, "llama.attention.head_count")) dst = &k.n_heads;
        else if (key_eq(key, kl, "llama.attention.head_count_kv")) dst = &k.n_kv_heads;
        else if (key_eq(key, kl, "llama.context_length")) dst = &k.seq_len;
        else if (key_eq(key, kl, "llama.rope.dimension_count")) dst = &k.rope_dim;
        if (dst && t == 4) {
            *dst = (int)cur_u(&c, 4);
        } else if (t == 6 && (key_eq(key, kl, "llama.rope.freq_base") ||
                              key_eq(key, kl, "llama.attention.layer_norm_rms_epsilon") ||
                              key_eq(key, kl, "llama.rope.scaling.factor") ||
                              key_eq(key, kl, "llama.rope.scale_linear"))) {
            uint32_t bits = (uint32_t)cur_u(&c, 4);
            float v;
            memcpy(&v, &bits, 4);
            if (key_eq(key, kl, "llama.rope.freq_base")) k.rope_freq_base = v;
            else if (key_eq(key, kl, "llama.attention.layer_norm_rms_epsilon")) k.rms_norm_eps = v;
            else if (key_eq(key, kl, "llama.rope.scaling.factor")) scal_factor = v;
            else scal_old = v;
        } else if (t == 8 && key_eq(key, kl, "llama.rope.scaling.type")) {
            uint64_t sl;
            const char *s = cur_str(&c, &sl);
            if (s) snprintf(scal_type, sizeof(scal_type), "%.*s", (int)sl, s);
        } else if (t == 4 && key_eq(key, kl, "general.alignment")) {
            align = (uint32_t)cur_u(&c, 4);
        } else if (t == 9 && key_eq(key, kl, "tokenizer.ggml.tokens")) {
            uint32_t et = (uint32_t)cur_u(&c, 4);
            uint64_t n = cur_u(&c, 8);
            k.vocab_size = (int)n;
            for (uint64_t j = 0; j < n && !c.bad; j++) cur_skip(&c, et);
        } else {
            cur_skip(&c, t);
        }
    }
    if (c.bad || !k.dim || !k.hidden_dim || !k.n_layers || !k.n_heads || !k.n_kv_heads ||
        !k.vocab_size || !k.seq_len) {
        seterr(err, cap, "missing metadata");
        orc_close(m);
        return NULL;
    }
    /* Defaults and linear RoPE scaling, src/checkpoint_gguf.c:694-737. */
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
        seterr(err, cap, "rope scaling");
        orc_close(m);
        return NULL;
    }

    m->t = (OrcTensor *)calloc(m->nt ? m->nt : 1, sizeof(OrcTensor));
    for (uint64_t i = 0; i < m->nt && !c.bad; i++) {
        uint64_t nl;
        const char *nm = cur_str(&c, &nl);
        if (nm == NULL || nl >= sizeof(m->t[i].name)) {
            c.bad = 1;
            break;
        }
        memcpy(m->t[i].name, nm, nl);
        m->t[i].ndim = (uint32_t)cur_u(&c, 4);
        if (m->t[i].ndim == 0 || m->t[i].ndim > 4) {
            c.bad = 1;
            break;
        }
        for (uint32_t d = 0; d < m->t[i].ndim; d++) m->t[i].dims[d] = cur_u(&c, 8);
        m->t[i].type = (uint32_t)cur_u(&c, 4);
        m->t[i].offset = cur_u(&c, 8);
    }
    if (c.bad) {
        seterr(err, cap, "bad tensor directory");
        orc_close(m);
        return NULL;
    }
    m->data_off = (c.pos + align - 1) / align * align;

    if (find_t(m, "rope_freqs.weight") != NULL) {
        seterr(err, cap, "rope_freqs unsupported");
        orc_close(m);
        return NULL;
    }
    const uint64_t dim = (uint64_t)k.dim, hid = (uint64_t)k.hidden_dim;
    const uint64_t kvd = dim / (uint64_t)k.n_heads * (uint64_t)k.n_kv_heads;
    OrcWeight onorm;
    if (!bind(m, "token_embd.weight", dim, (uint64_t)k.vocab_size, &m->embd) ||
        !bind(m, "output_norm.weight", dim, 0, &onorm)) {
        seterr(err, cap, "missing global tensor");
        orc_close(m);
        return NULL;
    }
    if (find_t(m, "output.weight") == NULL) {
        m->output = m->embd; /* tied, src/gguf_model.c:257-266 */
    } else if (!bind(m, "output.weight", dim, (uint64_t)k.vocab_size, &m->output)) {
        seterr(err, cap, "bad output tensor");
        orc_close(m);
        return NULL;
    }
    m->layers = (OrcLayer *)calloc((size_t)k.n_layers, sizeof(OrcLayer));
    m->norms = (float *)malloc((2 * (size_t)k.n_layers + 1) * dim * sizeof(float));
    for (int l = 0; l < k.n_layers; l++) {
        char nm[96];
        OrcLayer *L = &m->layers[l];
        OrcWeight an, fn;
#define B(suffix, cols, rows, dst) \
    (snprintf(nm, sizeof(nm), "blk.%d.%s", l, suffix), bind(m, nm, cols, rows, dst))
        if (!B("attn_norm.weight", dim, 0, &an) || !B("attn_q.weight", dim, dim, &L->wq) ||
            !B("attn_k.weight", dim, kvd, &L->wk) || !B("attn_v.weight", dim, kvd, &L->wv) ||
            !B("attn_output.weight", dim, dim, &L->wo) || !B("ffn_norm.weight", dim, 0, &fn) ||
            !B("ffn_gate.weight", dim, hid, &L->gate) || !B("ffn_up.weight", dim, hid, &L->up) ||
            !B("ffn_down.weight", hid, dim, &L->down)) {
            seterr(err, cap, "missing or malformed layer tensor");
            orc_close(m);
            return NULL;
        }
#undef B
        orc_dequantize_row(an.type, an.data, dim, m->norms + (2 * (size_t)l) * dim);
        orc_dequantize_row(fn.type, fn.data, dim, m->norms + (2 * (size_t)l + 1) * dim);
        L->attn_norm = m->norms + (2 * (size_t)l) * dim;
        L->ffn_norm = m->norms + (2 * (size_t)l + 1) * dim;
    }
    orc_dequantize_row(onorm.type, onorm.data, dim, m->norms + 2 * (size_t)k.n_layers * dim);

    m->file_context = k.seq_len;
    int capctx = max_context;
    if (capctx <= 0) capctx = k.seq_len < 4096 ? k.seq_len : 4096;
    if (capctx > k.seq_len) capctx = k.seq_len;
    k.seq_len = capctx;
    m->c = k;

    size_t cache = (size_t)k.n_layers * (size_t)k.seq_len * kvd;
    m->x = calloc(dim, 4);
    m->xb = calloc(dim, 4);
    m->xb2 = calloc(dim, 4);
    m->hb = calloc(hid, 4);
    m->hb2 = calloc(hid, 4);
    m->q = calloc(dim, 4);
    m->k = calloc(kvd, 4);
    m->v = calloc(kvd, 4);
    m->att = calloc((size_t)k.n_heads * (size_t)k.seq_len, 4);
    m->logits = calloc((size_t)k.vocab_size, 4);
    m->kc = calloc(cache, 4);
    m->vc = calloc(cache, 4);
    if (!m->x || !m->kc || !m->vc || !m->att || !m->logits) {
        seterr(err, cap, "out of memory");
        orc_close(m);
        return NULL;
    }
    return m;
}

void orc_close(OrcModel *m)
{
    if (m == NULL) return;
    free(m->file);
    free(m->t);
    free(m->layers);
    free(m->norms);
    free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2);
    free(m->q); free(m->k); free(m->v); free(m->att); free(m->logits);
    free(m->kc); free(m->vc);
    free(m);
}

/* Config as 7 ints (dim, hidden, layers, heads, kv_heads, vocab, seq_len),
 * rope_dim, and 3 floats (freq_base, eps, rope_scale). */
void orc_config(const OrcModel *m, int *ints8, float *floats3)
{
    const OrcConfig *c = &m->c;
    int v[8] = {c->dim, c->hidden_dim, c->n_layers, c->n_heads, c->n_kv_heads,
                c->vocab_size, c->seq_len, c->rope_dim};
    memcpy(ints8, v, sizeof(v));
    floats3[0] = c->rope_freq_base;
    floats3[1] = c->rms_norm_eps;
    floats3[2] = c->rope_scale;
}

/* Write K and V rows for (layer, pos) into the cache, as the forward pass
 * would have appended them (src/gguf_forward.c:220-226). Lets tests reach
 * long contexts without running every earlier position. */
int orc_kv_write(OrcModel *m, int layer, int pos, const float *k, const float *v)
{
    const OrcConfig *c = &m->c;
    size_t kvd = (size_t)(c->dim / c->n_heads * c->n_kv_heads);
    if (layer < 0 || layer >= c->n_layers || pos < 0 || pos >= c->seq_len) return 0;
    size_t off = ((size_t)layer * (size_t)c->seq_len + (size_t)pos) * kvd;
    memcpy(m->kc + off, k, kvd * 4);
    memcpy(m->vc + off, v, kvd * 4);
    return 1;
}

/* Not in the reference (its cache is float, README.md:194): the variant
 * whose appended K/V entries are rounded to IEEE binary16, round to nearest
 * even (C's _Float16 conversion), and read back exactly. The rest of the
 * forward is unchanged. */
int orc_set_kv_half(OrcModel *m, int on)
{
    if (m == NULL) return 0;
    m->kv_half = on != 0;
    return 1;
}

static void kv_append(float *dst, const float *src, int n, int half)
{
    if (!half) {
        memcpy(dst, src, (size_t)n * 4);
        return;
    }
    for (int i = 0; i < n; i++) dst[i] = (float)(_Float16)src[i];
}

/* rmsnorm_eps, src/gguf_forward.c:24-40. */
static void rmsnorm(float *o, const float *x, const float *w, int n, float eps)
{
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss /= (float)n;
    ss += eps;
    ss = 1.0f / sqrtf(ss);
    for (int i = 0; i < n; i++) o[i] = w[i] * (ss * x[i]);
}

/* rope_head, src/gguf_forward.c:50-66. */
static void rope(float *v, int rope_dim, int pos, float base, float scale)
{
    const float p = (float)pos / scale;
    for (int i = 0; i < rope_dim; i += 2) {
        const float fr = 1.0f / powf(base, (float)i / (float)rope_dim);
        const float a = p * fr;
        const float c = cosf(a), s = sinf(a);
        const float v0 = v[i], v1 = v[i + 1];
        v[i] = v0 * c - v1 * s;
        v[i + 1] = v0 * s + v1 * c;
    }
}

/* softmax, src/transformer.c:85-109. */
static void softmax(float *x, int n)
{
    if (n <= 0) return;
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* The RoPE angle table entries (cos, sin) used at `pos`, in the order
 * rope() evaluates them: out[2*(i/2)] = cosf, out[2*(i/2)+1] = sinf. */
void orc_rope_table(const OrcModel *m, int pos, float *out)
{
    const OrcConfig *c = &m->c;
    const float p = (float)pos / c->rope_scale;
    for (int i = 0; i < c->rope_dim; i += 2) {
        const float fr = 1.0f / powf(c->rope_freq_base, (float)i / (float)c->rope_dim);
        const float a = p * fr;
        out[i] = cosf(a);
        out[i + 1] = sinf(a);
    }
}

/* gguf_forward, src/gguf_forward.c:159-313. */
float *orc_forward(OrcModel *m, int token, int pos)
{
    const OrcConfig *p = &m->c;
    if (m == NULL || token < 0 || token >= p->vocab_size || pos < 0 || pos >= p->seq_len) {
        return NULL;
    }
    const int dim = p->dim, hid = p->hidden_dim;
    const int hs = dim / p->n_heads;
    const int kvd = hs * p->n_kv_heads;
    const int kvmul = p->n_heads / p->n_kv_heads;
    const size_t seq = (size_t)p->seq_len;
    const float scale = 1.0f / sqrtf((float)hs);
    const float eps = p->rms_norm_eps;

    orc_dequantize_row(m->embd.type, m->embd.data + (size_t)token * m->embd.row_bytes,
                       (uint64_t)dim, m->x);

    for (int l = 0; l < p->n_layers; l++) {
        const OrcLayer *L = &m->layers[l];
        const size_t lc = (size_t)l * seq * (size_t)kvd;

        rmsnorm(m->xb, m->x, L->attn_norm, dim, eps);
        orc_matvec(L->wq.type, L->wq.data, L->wq.rows, L->wq.cols, m->xb, m->q);
        orc_matvec(L->wk.type, L->wk.data, L->wk.rows, L->wk.cols, m->xb, m->k);
        orc_matvec(L->wv.type, L->wv.data, L->wv.rows, L->wv.cols, m->xb, m->v);
        for (int h = 0; h < p->n_heads; h++) {
            rope(m->q + (size_t)h * hs, p->rope_dim, pos, p->rope_freq_base, p->rope_scale);
        }
        for (int h = 0; h < p->n_kv_heads; h++) {
            rope(m->k + (size_t)h * hs, p->rope_dim, pos, p->rope_freq_base, p->rope_scale);
        }
        kv_append(m->kc + lc + (size_t)pos * kvd, m->k, kvd, m->kv_half);
        kv_append(m->vc + lc + (size_t)pos * kvd, m->v, kvd, m->kv_half);

        for (int h = 0; h < p->n_heads; h++) {
            const float *qh = m->q + (size_t)h * hs;
            float *att = m->att + (size_t)h * seq;
            const size_t kvo = (size_t)(h / kvmul) * (size_t)hs;
            for (int t = 0; t <= pos; t++) {
                const float *kk = m->kc + lc + (size_t)t * kvd + kvo;
                float s = 0.0f;
                for (int i = 0; i < hs; i++) s += qh[i] * kk[i];
                att[t] = s * scale;
            }
            softmax(att, pos + 1);
            float *o = m->xb + (size_t)h * hs;
            for (int i = 0; i < hs; i++) o[i] = 0.0f;
            for (int t = 0; t <= pos; t++) {
                const float *vv = m->vc + lc + (size_t)t * kvd + kvo;
                const float a = att[t];
                for (int i = 0; i < hs; i++) o[i] += a * vv[i];
            }
        }
        orc_matvec(L->wo.type, L->wo.data, L->wo.rows, L->wo.cols, m->xb, m->xb2);
        for (int i = 0; i < dim; i++) m->x[i] += m->xb2[i];

        rmsnorm(m->xb, m->x, L->ffn_norm, dim, eps);
        orc_matvec(L->gate.type, L->gate.data, L->gate.rows, L->gate.cols, m->xb, m->hb);
        orc_matvec(L->up.type, L->up.data, L->up.rows, L->up.cols, m->xb, m->hb2);
        for (int i = 0; i < hid; i++) {
            const float g = m->hb[i];
            m->hb[i] = (g / (1.0f + expf(-g))) * m->hb2[i];
        }
        orc_matvec(L->down.type, L->down.data, L->down.rows, L->down.cols, m->hb, m->xb);
        for (int i = 0; i < dim; i++) m->x[i] += m->xb[i];
    }
    rmsnorm(m->x, m->x, m->norms + 2 * (size_t)p->n_layers * dim, dim, eps);
    orc_matvec(m->output.type, m->output.data, m->output.rows, m->output.cols, m->x, m->logits);
    return m->logits;
}

/* sampler_greedy, src/sampler.c:39-52: first maximum wins; -1 if none. */
int orc_greedy(const float *logits, int n)
{
    if (logits == NULL || n <= 0) return -1;
    int best = -1;
    float bv = 0.0f;
    for (int i = 0; i < n; i++) {
        if (!isfinite(logits[i])) return -1;
        if (best < 0 || logits[i] > bv) {
            best = i;
            bv = logits[i];
        }
    }
    return best;
}
