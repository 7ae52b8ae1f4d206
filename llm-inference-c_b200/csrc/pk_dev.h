/*
 * pk_dev.h - the internal C ABI between the C11 host engine (engine.c) and
 * the CUDA side (pk_device.cu). Plain C types only.
 */
#ifndef PK_DEV_H
#define PK_DEV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One weight tensor inside the device weight arena. */
typedef struct {
    uint32_t type;      /* GGML type id */
    uint64_t rows;      /* ne1 (1 for vectors) */
    uint64_t cols;      /* ne0 */
    uint64_t row_bytes;
    uint64_t offset;    /* byte offset of row 0 inside the arena */
} PkdTensor;

/* Most ranks of one tensor-parallel group. */
#define PKD_TP_MAX 8

/* Tensor-parallel placement of one rank (world 1: everything local). Query
 * and KV heads, the hidden slice (gate/up rows = down columns, whole
 * quant blocks) and the output's vocabulary rows are this rank's; the
 * residual stream x is replicated, and rank r reduces elements
 * [own0[r], own0[r] + own[r]) of each all-reduce. */
typedef struct {
    int rank, world;
    int q_head0, q_heads;
    int kv_head0, kv_heads;
    int hid0, hid, hid_max;
    int voc0, voc;
    int own0[PKD_TP_MAX], own[PKD_TP_MAX];
    int own_max;
} PkdTp;

typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, rope_dim;
    int head_size;              /* dim / the model's head count */
    PkdTp tp;                   /* n_heads, n_kv_heads, hidden_dim above are this rank's */
    float rms_eps;
    float att_scale;            /* 1/sqrtf(head_size), computed as the reference does */
    PkdTensor embd, output;
    const PkdTensor *wq, *wk, *wv, *wo, *gate, *up, *down; /* n_layers each */
    const PkdTensor *attn_norm, *ffn_norm;                  /* n_layers each, decoded on the device */
    PkdTensor output_norm;
    const float *rope_cs;       /* host: seq_len * rope_dim floats, (cos, sin) pairs */
    int kv_half;                /* KV cache entries: IEEE half (1) or float (0) */
} PkdModel;

typedef struct PkdCtx PkdCtx;

/* Device context for one handle on `device`. NULL + message on failure. */
PkdCtx *pkd_create(int device, uint64_t arena_bytes, char *err, size_t cap);
void pkd_destroy(PkdCtx *ctx);

/* Copy `bytes` host bytes to arena offset `offset` (through pinned staging). */
int pkd_upload(PkdCtx *ctx, uint64_t offset, const void *src, uint64_t bytes, char *err, size_t cap);

/* Allocate run state (KV cache, activations), upload norms and the RoPE
 * table, and - for a single rank - build and capture the decode step. A
 * tensor-parallel rank builds its step in pkd_tp_connect. */
int pkd_build(PkdCtx *ctx, const PkdModel *m, char *err, size_t cap);

/* Tensor parallel: this rank's exchange-buffer handle (64 bytes, a CUDA IPC
 * memory handle) for the other ranks. */
int pkd_tp_handle(PkdCtx *ctx, void *out64, char *err, size_t cap);

/* Tensor parallel: map the other ranks' exchange buffers (world handles of
 * 64 bytes in rank order), then build and capture the decode step. */
int pkd_tp_connect(PkdCtx *ctx, const void *handles, char *err, size_t cap);

/* One decode step. Returns host (pinned) logits owned by ctx, or NULL on a
 * device error (ctx then stays failed). */
float *pkd_forward(PkdCtx *ctx, int token, int pos);

/* One decode step returning the greedy token (device argmax, lowest index
 * on ties); -1 if a logit is not finite; -2 on a device error. */
int pkd_forward_greedy(PkdCtx *ctx, int token, int pos);

/* n greedy steps fed back on the device (token, pos), (argmax, pos+1), ...
 * without host round trips; out receives the n generated tokens (-1 where
 * a logit was not finite) and device_ms the CUDA-event time of the n graph
 * replays. Returns 1 on success. */
int pkd_generate_greedy(PkdCtx *ctx, int token, int pos, int n, int *out, float *device_ms);

/* With POCKET_CUDA_TRACE=1: the %globaltimer stamps (ns) of the last
 * persistent step - CTA 0's start, then for each phase: after staging x,
 * after the phase's work, at the phase's end; then for every CTA and phase:
 * after staging x, after the work. Returns the count. */
int pkd_trace(PkdCtx *ctx, unsigned long long *out, int cap);

/* Write positions [pos0, pos0 + npos) of layer `layer` of the decode-step
 * KV cache: k and v are npos rows of this rank's kv_dim floats each (stored
 * as the cache holds them: float, or rounded to half). Synchronous. */
int pkd_kv_write(PkdCtx *ctx, int layer, int pos0, int npos, const float *k, const float *v, char *err,
                 size_t cap);

/* Last device error message ("" if none). */
const char *pkd_error(const PkdCtx *ctx);

/* Kernel launches per decode step (2 with the cooperative step kernel,
 * phases + 1 otherwise). */
int pkd_launches_per_step(const PkdCtx *ctx);

/* What the batched step (pk_batch.cu) reads from a built single-GPU
 * context: the stream, the weight arena, the decoded norms
 * ([2 * n_layers + 1][dim]: attention and FFN norm of each layer, then the
 * output norm), the RoPE table on the device ([seq_len][rope_dim]) and the
 * model (tensor tables owned by the context). */
typedef struct {
    int device;
    void *stream;
    const uint8_t *arena;
    const float *norms;
    const float *rope_cs;
    const PkdModel *model;
    void *kc, *vc;  /* the decode step's KV cache ([layer][position][kv_dim]) */
    /* tensor parallel (world > 1, after pkd_tp_connect): every rank's
     * exchange buffer (64-bit tagged words, mapped here), where the batched
     * step's exchange region starts in it (bx, in words) and how many words
     * one rank's part of a slot holds (bx_len); [2 slots][world][bx_len] */
    int rank, world;
    uint64_t *peers[PKD_TP_MAX];
    uint64_t bx, bx_len;
} PkdView;

/* 0 for an unbuilt context or a tensor-parallel rank before pkd_tp_connect. */
int pkd_view(PkdCtx *ctx, PkdView *out);

/* Batched decode: one step for up to 64 independent sequences that share
 * one pass over the weights (pk_batch.cu). */
typedef struct PkbCtx PkbCtx;

/* Run state for max_seqs sequences (each a KV cache of the model's
 * seq_len) on ctx's device and stream. NULL + message on failure. */
PkbCtx *pkb_create(PkdCtx *ctx, int max_seqs, char *err, size_t cap);

/* A one-sequence batched state whose KV cache IS the decode step's (the
 * layout of sequence 0 of a batched cache): prompt chunks run through the
 * batched step and land where engine_forward reads them. */
PkbCtx *pkb_create_prefill(PkdCtx *ctx, char *err, size_t cap);
void pkb_destroy(PkbCtx *b);

/* Sequence seq_ids[i] takes tokens[i] at position pos[i], i < n. next[i]
 * receives the greedy token (-1 when a logit is not finite); logits (n x
 * vocab floats, host) when not NULL. Arguments are checked by the caller.
 * Returns 1, or 0 on a device error (message in pkb_error). */
int pkb_step(PkbCtx *b, const int *tokens, const int *pos, const int *seq_ids, int n, int *next, float *logits);
const char *pkb_error(const PkbCtx *b);

/* pkd_kv_write for sequence `seq` of the batched state. */
int pkb_kv_write(PkbCtx *b, int seq, int layer, int pos0, int npos, const float *k, const float *v, char *err,
                 size_t cap);

#ifdef __cplusplus
}
#endif

#endif
