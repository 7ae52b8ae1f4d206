/*
 * vocab.c - fill the Tokenizer record returned by engine_tokenizer().
 *
 * The record is what the reference's text tokenizer reads, so it is filled
 * with the same content the reference's loaders produce:
 *   pk_vocab_load_gguf : src/gguf_tokenizer.c:225-510 (SentencePiece "llama"
 *                        metadata: U+2581 -> ' ', byte tokens, special
 *                        tokens, -inf scores for tokens merges may not
 *                        build, score rebuild when all scores are equal);
 *   pk_vocab_load_bin  : src/tokenizer.c:55-190 (llama2.c tokenizer.bin).
 * Text encoding / decoding itself is outside the decode path.
 */
#define _POSIX_C_SOURCE 200809L
#include "tokenizer.h"

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

enum { TT_NORMAL = 1, TT_UNKNOWN = 2, TT_CONTROL = 3, TT_USER = 4, TT_UNUSED = 5, TT_BYTE = 6 };

void tokenizer_free(Tokenizer *t)
{
    if (t == NULL) return;
    if (t->vocab != NULL) {
        for (size_t i = 0; i < t->vocab_size; i++) free(t->vocab[i]);
    }
    free(t->vocab);
    free(t->scores);
    free(t->sorted_vocab);
    free(t->special_ids);
    memset(t, 0, sizeof(*t));
}

static void seterr(char *e, size_t cap, const char *msg)
{
    if (e != NULL && cap > 0) snprintf(e, cap, "%s", msg);
}

typedef struct {
    const unsigned char *p;
    size_t n, pos;
    int bad;
} Rd;

static uint64_t get(Rd *r, int bytes)
{
    if (r->bad || (size_t)bytes > r->n - r->pos) {
        r->bad = 1;
        return 0;
    }
    uint64_t v = 0;
    for (int i = 0; i < bytes; i++) v |= (uint64_t)r->p[r->pos + (size_t)i] << (8 * i);
    r->pos += (size_t)bytes;
    return v;
}

static const char *get_str(Rd *r, uint64_t *len)
{
    *len = get(r, 8);
    if (r->bad || *len > r->n - r->pos) {
        r->bad = 1;
        return NULL;
    }
    const char *s = (const char *)r->p + r->pos;
    r->pos += (size_t)*len;
    return s;
}

static size_t scalar(uint32_t t)
{
    static const size_t sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    return t < 13 ? sz[t] : 0;
}

static void skip(Rd *r, uint32_t t)
{
    uint64_t len;
    if (t == 8) {
        (void)get_str(r, &len);
    } else if (t == 9) {
        const uint32_t et = (uint32_t)get(r, 4);
        const uint64_t n = get(r, 8);
        if (et == 9) {
            r->bad = 1;
        } else if (et == 8) {
            for (uint64_t i = 0; i < n && !r->bad; i++) skip(r, 8);
        } else {
            const size_t s = scalar(et);
            if (s == 0 || n > (r->n - r->pos) / s) r->bad = 1;
            else r->pos += (size_t)n * s;
        }
    } else {
        const size_t s = scalar(t);
        if (s == 0 || s > r->n - r->pos) r->bad = 1;
        else r->pos += s;
    }
}

static int keyeq(const char *k, uint64_t n, const char *s)
{
    return strlen(s) == n && memcmp(k, s, (size_t)n) == 0;
}

/* A piece with every U+2581 (E2 96 81) turned into ' '. */
static char *piece_copy(const char *s, uint64_t n)
{
    char *o = (char *)malloc((size_t)n + 1);
    size_t k = 0;
    if (o == NULL) return NULL;
    for (uint64_t i = 0; i < n; i++) {
        if (i + 2 < n && (unsigned char)s[i] == 0xE2 && (unsigned char)s[i + 1] == 0x96 &&
            (unsigned char)s[i + 2] == 0x81) {
            o[k++] = ' ';
            i += 2;
        } else {
            o[k++] = s[i];
        }
    }
    o[k] = '\0';
    return o;
}

static int by_text(const void *a, const void *b)
{
    return strcmp(((const TokenizerIndex *)a)->text, ((const TokenizerIndex *)b)->text);
}

static int sort_and_bytes(Tokenizer *t)
{
    t->sorted_vocab = (TokenizerIndex *)malloc(t->vocab_size * sizeof(TokenizerIndex));
    if (t->sorted_vocab == NULL) return 0;
    for (size_t i = 0; i < t->vocab_size; i++) {
        t->sorted_vocab[i].text = t->vocab[i];
        t->sorted_vocab[i].id = (int)i;
    }
    qsort(t->sorted_vocab, t->vocab_size, sizeof(TokenizerIndex), by_text);
    for (int i = 0; i < 256; i++) {
        t->byte_pieces[2 * i] = (unsigned char)i;
        t->byte_pieces[2 * i + 1] = '\0';
    }
    return 1;
}

static int read_int(Rd *r, uint32_t type, int64_t *out)
{
    switch (type) {
    case 4: *out = (int64_t)(uint32_t)get(r, 4); return !r->bad;
    case 5: *out = (int64_t)(int32_t)(uint32_t)get(r, 4); return !r->bad;
    case 10: case 11: *out = (int64_t)get(r, 8); return !r->bad;
    default: skip(r, type); return 0;
    }
}

int pk_vocab_load_gguf(Tokenizer *t, const unsigned char *file, size_t size, char *err, size_t cap)
{
    const char *msg = "Invalid or truncated GGUF tokenizer metadata.";
    int32_t *types = NULL;
    size_t n_types = 0, n_scores = 0;
    int have_model = 0;
    int64_t bos = 1, eos = 2;
    memset(t, 0, sizeof(*t));
    Rd r = {file, size, 4, 0};
    if (size < 24 || memcmp(file, "GGUF", 4) != 0) {
        msg = "Not a GGUF file.";
        goto fail;
    }
    {
        const uint32_t ver = (uint32_t)get(&r, 4);
        if (ver < 2 || ver > 3) {
            msg = "Unsupported GGUF version.";
            goto fail;
        }
    }
    (void)get(&r, 8);
    const uint64_t nkv = get(&r, 8);
    for (uint64_t k = 0; k < nkv && !r.bad; k++) {
        uint64_t kl;
        const char *key = get_str(&r, &kl);
        const uint32_t type = (uint32_t)get(&r, 4);
        if (key == NULL || r.bad) break;
        if (keyeq(key, kl, "tokenizer.ggml.model")) {
            uint64_t ml;
            const char *mv = type == 8 ? get_str(&r, &ml) : NULL;
            if (mv == NULL || ml != 5 || memcmp(mv, "llama", 5) != 0) {
                msg = "Only SentencePiece ('llama') GGUF tokenizers are supported.";
                goto fail;
            }
            have_model = 1;
        } else if (keyeq(key, kl, "tokenizer.ggml.tokens")) {
            if (type != 9 || get(&r, 4) != 8) goto fail;
            const uint64_t n = get(&r, 8);
            if (n < 1 || n > (uint64_t)INT32_MAX || n > (r.n - r.pos) / 8) goto fail;
            t->vocab_size = (size_t)n;
            t->vocab = (char **)calloc((size_t)n, sizeof(char *));
            if (t->vocab == NULL) {
                msg = "Memory allocation failed.";
                goto fail;
            }
            for (uint64_t i = 0; i < n; i++) {
                uint64_t pl;
                const char *pc = get_str(&r, &pl);
                if (pc == NULL || memchr(pc, '\0', (size_t)pl) != NULL) goto fail;
                t->vocab[i] = piece_copy(pc, pl);
                if (t->vocab[i] == NULL) {
                    msg = "Memory allocation failed.";
                    goto fail;
                }
                const size_t len = strlen(t->vocab[i]);
                if (len > t->max_token_length) t->max_token_length = len;
            }
        } else if (keyeq(key, kl, "tokenizer.ggml.scores")) {
            if (type != 9 || get(&r, 4) != 6) goto fail;
            const uint64_t n = get(&r, 8);
            if (n > (r.n - r.pos) / 4) goto fail;
            free(t->scores);
            t->scores = (float *)malloc((size_t)(n ? n : 1) * sizeof(float));
            if (t->scores == NULL) {
                msg = "Memory allocation failed.";
                goto fail;
            }
            for (uint64_t i = 0; i < n; i++) {
                const uint32_t bits = (uint32_t)get(&r, 4);
                memcpy(&t->scores[i], &bits, 4);
            }
            n_scores = (size_t)n;
        } else if (keyeq(key, kl, "tokenizer.ggml.token_type")) {
            if (type != 9 || get(&r, 4) != 5) goto fail;
            const uint64_t n = get(&r, 8);
            if (n > (r.n - r.pos) / 4) goto fail;
            free(types);
            types = (int32_t *)malloc((size_t)(n ? n : 1) * sizeof(int32_t));
            if (types == NULL) {
                msg = "Memory allocation failed.";
                goto fail;
            }
            for (uint64_t i = 0; i < n; i++) types[i] = (int32_t)(uint32_t)get(&r, 4);
            n_types = (size_t)n;
        } else if (keyeq(key, kl, "tokenizer.ggml.bos_token_id")) {
            if (!read_int(&r, type, &bos)) goto fail;
        } else if (keyeq(key, kl, "tokenizer.ggml.eos_token_id")) {
            if (!read_int(&r, type, &eos)) goto fail;
        } else {
            skip(&r, type);
        }
    }
    if (r.bad) goto fail;
    if (!have_model || t->vocab == NULL || t->scores == NULL) {
        msg = "GGUF file has no SentencePiece tokenizer metadata.";
        goto fail;
    }
    {
        const size_t n = t->vocab_size;
        if (n_scores != n || (types != NULL && n_types != n)) {
            msg = "Tokenizer arrays have different lengths.";
            goto fail;
        }
        if (bos < 0 || (size_t)bos >= n || eos < 0 || (size_t)eos >= n) {
            msg = "BOS/EOS token ID is outside the vocabulary.";
            goto fail;
        }
        t->bos_id = (int)bos;
        t->eos_id = (int)eos;
        /* Rebuild scores from token order when normal scores are all equal. */
        float lo = INFINITY, hi = -INFINITY;
        for (size_t i = 0; i < n; i++) {
            if ((types ? types[i] : TT_NORMAL) == TT_NORMAL) {
                if (t->scores[i] < lo) lo = t->scores[i];
                if (t->scores[i] > hi) hi = t->scores[i];
            }
        }
        if (lo == hi) {
            for (size_t i = 0; i < n; i++) {
                const char *pc = t->vocab[i];
                int spaces = pc[0] != '\0';
                for (const char *q = pc; *q; q++) {
                    if (*q != ' ') {
                        spaces = 0;
                        break;
                    }
                }
                t->scores[i] = spaces ? -1e9f : -(float)i;
            }
            t->scores_reconstructed = 1;
        }
        for (int i = 0; i < 256; i++) t->byte_ids[i] = -1;
        t->special_ids = (int *)malloc(n * sizeof(int));
        if (t->special_ids == NULL) {
            msg = "Memory allocation failed.";
            goto fail;
        }
        for (size_t i = 0; i < n; i++) {
            const char *pc = t->vocab[i];
            const int32_t ty = types ? types[i] : TT_NORMAL;
            if (!isfinite(t->scores[i])) {
                msg = "Tokenizer score is not finite.";
                goto fail;
            }
            const int byte_name = strlen(pc) == 6 && pc[0] == '<' && pc[1] == '0' && pc[2] == 'x' && pc[5] == '>';
            if (byte_name && (types == NULL || ty == TT_BYTE)) {
                char hx[3] = {pc[3], pc[4], '\0'};
                char *end = NULL;
                const unsigned long v = strtoul(hx, &end, 16);
                if (end == hx + 2 && v < 256) t->byte_ids[v] = (int)i;
            }
            if (ty == TT_UNKNOWN || ty == TT_CONTROL || ty == TT_UNUSED || ty == TT_BYTE ||
                (types == NULL && byte_name)) {
                t->scores[i] = -INFINITY;
            }
            if ((ty == TT_UNKNOWN || ty == TT_CONTROL || ty == TT_USER) && pc[0] != '\0') {
                t->special_ids[t->n_special++] = (int)i;
            }
        }
        if (!sort_and_bytes(t)) {
            msg = "Memory allocation failed.";
            goto fail;
        }
    }
    free(types);
    if (err && cap) err[0] = '\0';
    return 0;
fail:
    seterr(err, cap, msg);
    free(types);
    tokenizer_free(t);
    return -1;
}

int pk_vocab_load_bin(Tokenizer *t, const char *path, size_t vocab_size, char *err, size_t cap)
{
    memset(t, 0, sizeof(*t));
    if (path == NULL || path[0] == '\0' || vocab_size < 259 || vocab_size > (size_t)INT32_MAX) {
        seterr(err, cap, "Invalid tokenizer arguments.");
        return -1;
    }
    FILE *f = fopen(path, "rb");
    if (f == NULL) {
        seterr(err, cap, "Cannot open tokenizer file.");
        return -1;
    }
    uint32_t maxlen = 0;
    if (fread(&maxlen, 4, 1, f) != 1 || maxlen == 0 || maxlen > 1048576u) {
        fclose(f);
        seterr(err, cap, "Invalid tokenizer header.");
        return -1;
    }
    t->vocab_size = vocab_size;
    t->max_token_length = maxlen;
    t->vocab = (char **)calloc(vocab_size, sizeof(char *));
    t->scores = (float *)calloc(vocab_size, sizeof(float));
    if (t->vocab == NULL || t->scores == NULL) {
        fclose(f);
        tokenizer_free(t);
        seterr(err, cap, "Memory allocation failed.");
        return -1;
    }
    for (size_t i = 0; i < vocab_size; i++) {
        uint32_t len = 0;
        if (fread(&t->scores[i], 4, 1, f) != 1 || !isfinite(t->scores[i]) || fread(&len, 4, 1, f) != 1 ||
            len == 0 || len > maxlen) {
            fclose(f);
            tokenizer_free(t);
            seterr(err, cap, "Tokenizer file is truncated or contains invalid entries.");
            return -1;
        }
        t->vocab[i] = (char *)malloc((size_t)len + 1);
        if (t->vocab[i] == NULL || fread(t->vocab[i], 1, len, f) != len) {
            fclose(f);
            tokenizer_free(t);
            seterr(err, cap, "Tokenizer file is truncated.");
            return -1;
        }
        t->vocab[i][len] = '\0';
        if (memchr(t->vocab[i], '\0', len) != NULL) {
            fclose(f);
            tokenizer_free(t);
            seterr(err, cap, "Tokenizer entry contains an embedded NUL byte.");
            return -1;
        }
    }
    const int trailing = fgetc(f) != EOF;
    fclose(f);
    if (trailing) {
        tokenizer_free(t);
        seterr(err, cap, "Tokenizer file has unexpected trailing data.");
        return -1;
    }
    if (!sort_and_bytes(t)) {
        tokenizer_free(t);
        seterr(err, cap, "Memory allocation failed.");
        return -1;
    }
    if (strcmp(t->vocab[1], "\n<s>\n") != 0 || strcmp(t->vocab[2], "\n</s>\n") != 0) {
        tokenizer_free(t);
        seterr(err, cap, "Tokenizer special-token IDs do not match expected format.");
        return -1;
    }
    t->bos_id = 1;
    t->eos_id = 2;
    for (int b = 0; b < 256; b++) t->byte_ids[b] = b + 3;
    return 0;
}
