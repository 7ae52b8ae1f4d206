/*
 * engine_ext.h - additive entry points of the B200 engine. They have no
 * counterpart in the reference's engine.h; existing signatures are
 * unchanged.
 */
#ifndef ENGINE_EXT_H
#define ENGINE_EXT_H

#include "engine.h"

#ifdef __cplusplus
extern "C" {
#endif

/* engine_open on an explicit CUDA device (engine_open uses
 * POCKET_CUDA_DEVICE, default 0). */
LLMModel *engine_open_device(const LLMOptions *options, int device,
                             char *error, size_t error_capacity);

/* One decode step that returns the greedy token instead of the logits:
 * the argmax runs on the device (lowest index wins ties, as the
 * reference's sampler_greedy, src/sampler.c:39-52) and only 4 bytes come
 * back. Returns -1 if any logit is not finite, -2 for invalid arguments or
 * a device error (same validity rules as engine_forward). */
int engine_forward_greedy(LLMModel *model, int token, int pos);

/* n greedy decode steps run back to back on the device: step i feeds the
 * argmax of step i-1 (the first step feeds `token`) at position pos + i,
 * with no host round trip in between. out_tokens receives the n generated
 * tokens (-1 where a logit was not finite; generation then continues from
 * token 0). device_ms (optional) receives the CUDA-event time of the n
 * steps. Requires pos + n <= seq_len. Returns 1 on success, 0 on invalid
 * arguments or a device error. */
int engine_generate_greedy(LLMModel *model, int token, int pos, int n,
                           int *out_tokens, float *device_ms);

/* Tracing: when the handle was opened with POCKET_CUDA_TRACE=1, copies the
 * device timestamps (ns, %globaltimer) of the last decode step into out and
 * returns how many were written (0 when tracing is off). First CTA 0's: the
 * step's start, then for each of its P = 5 * n_layers + 1 phases the time
 * after staging the input vector, after the phase's work and again at the
 * phase's end (3P + 1 words). Then, for every CTA b of the step's grid in
 * order, 2P words: per phase, after staging and after the work. */
int engine_trace(LLMModel *model, unsigned long long *out, int cap);

/* Message of the last device error of this handle ("" if none). */
const char *engine_last_error(const LLMModel *model);

/* Bytes of packed weights resident on the device. */
size_t engine_weight_bytes(const LLMModel *model);

/* ---- Tensor parallelism over the GPUs of one box -------------------
 *
 * One process per GPU; the ranks' decode kernels exchange partial sums
 * over NVLink peer memory inside the decode step (two all-reduces per
 * layer, no library collective). Query/KV heads, the FFN hidden slice and
 * the output's vocabulary rows are split over the ranks; the embedding,
 * the norms and the residual stream are replicated. Every rank's
 * engine_forward returns the full logits, every rank's greedy token is the
 * global argmax. Usage, on each rank:
 *
 *   m = engine_open_tp(&opts, device, rank, world, err, cap);
 *   engine_tp_handle(m, mine);            // 64 bytes
 *   ... all-gather the ranks' 64-byte handles in rank order ...
 *   engine_tp_connect(m, all, err, cap);  // then decode as usual, every
 *                                         // rank feeding the same tokens
 */

/* Placement of one rank. */
typedef struct {
    int q_head0, q_heads;   /* query heads */
    int kv_head0, kv_heads; /* KV heads (shared by ranks when world > n_kv_heads) */
    int hid0, hid;          /* ffn_gate / ffn_up rows = ffn_down columns */
    int voc0, voc;          /* output (logits) rows */
    int own0, own;          /* residual-stream elements this rank reduces */
} EngineTpPlan;

/* The placement of rank `rank` of `world` (1..8) for a model of these
 * dimensions; wo_block and down_block are the block widths (weights per
 * block, e.g. 256 for Q4_K) of attn_output and ffn_down. Returns 1, or 0
 * with a message when the model cannot be split that way. */
int engine_tp_plan(int dim, int hidden_dim, int n_heads, int n_kv_heads, int vocab_size,
                   int wo_block, int down_block, int rank, int world, EngineTpPlan *out,
                   char *error, size_t error_capacity);

/* engine_open_device for rank `rank` of a tensor-parallel group of
 * `world` GPUs: loads only this rank's slices. The handle decodes after
 * engine_tp_connect. world 1 is engine_open_device. */
LLMModel *engine_open_tp(const LLMOptions *options, int device, int rank, int world,
                         char *error, size_t error_capacity);

/* This rank's 64-byte exchange handle. Returns 1, or 0 for a handle that is
 * not tensor-parallel. */
int engine_tp_handle(LLMModel *model, void *out64);

/* Connect the ranks: `handles` holds world 64-byte handles in rank order.
 * Returns 1, or 0 with a message (the handle then stays unusable). */
int engine_tp_connect(LLMModel *model, const void *handles, char *error, size_t error_capacity);

/* Kernel launches one decode step makes: 2 in the default mode (the
 * cooperative step kernel and the one-thread token kernel), one per phase
 * plus one (5 * n_layers + 2) with POCKET_CUDA_PERSISTENT=0 or when the GPU
 * cannot co-schedule the step kernel; 0 for a NULL handle. */
int engine_launches_per_step(const LLMModel *model);

/* ---- Batched decode (additive; the reference decodes one sequence) --
 * Up to ENGINE_BATCH_MAX independent sequences decode together, sharing
 * one pass over the weights per step: Q4_K, Q5_K and Q6_K matrices on the
 * tensor cores, the other formats on CUDA cores. Each sequence has its own
 * KV cache of the model's context length, separate from the one
 * engine_forward uses. Runs on one GPU or on a tensor-parallel group (all
 * ranks making the same calls). */
#define ENGINE_BATCH_MAX 64

/* Allocate the batched state for max_seqs sequences (1..64), dropping any
 * previous one. On a tensor-parallel rank (after engine_tp_connect) every
 * rank of the group opens the same state: each rank keeps the KV heads of
 * its own query heads for every sequence. Returns 1, or 0 with a message in
 * error. */
int engine_batch_open(LLMModel *model, int max_seqs, char *error, size_t error_capacity);

/* One step over n <= 64 rows: sequence seq_ids[i] consumes tokens[i] at
 * position pos[i] (seq_ids below max_seqs; tokens in the vocabulary;
 * positions below the context length; each (sequence, position) at most
 * once per call; no gaps: positions 0 .. pos[i] - 1 of the sequence were
 * filled by earlier calls, by engine_kv_write or by rows of this call),
 * exactly as engine_forward(tokens[i], pos[i]) would for that sequence
 * alone. Rows of one sequence at consecutive positions form a
 * prompt chunk (prefill): every row's keys and values are appended before
 * any row attends, so row i sees the sequence's positions 0 .. pos[i].
 * next_tokens[i] receives the greedy token of row i (device argmax, lowest
 * index on ties; -1 when a logit is not finite); logits, when not NULL, the
 * n x vocab_size logits. Tensor parallel: every rank of the group makes the
 * same call (the same rows, and logits given on all ranks or on none); the
 * ranks add their heads' and hidden slices' partial sums after Wo and
 * ffn_down over NVLink, pick the greedy tokens over their vocabulary slices,
 * and each rank returns the same tokens (and full logits). Returns 1, or 0
 * on bad arguments or a device error (engine_last_error). */
int engine_forward_batch(LLMModel *model, const int *tokens, const int *pos, const int *seq_ids, int n,
                         int *next_tokens, float *logits);

/* A prompt of n tokens at positions pos0 .. pos0 + n - 1 of the cache
 * engine_forward uses, in chunks of up to 64 rows through the batched step
 * (the dense matmuls on the tensor cores), instead of n engine_forward calls
 * (the reference feeds prompts one token at a time, src/pocket.c:294-301).
 * Every position's K/V is appended before its chunk attends, so position i
 * sees positions 0 .. i: afterwards engine_forward / engine_generate_greedy
 * continue at pos0 + n exactly as after n engine_forward calls (within
 * float rounding). Positions below pos0 hold what earlier calls wrote.
 * last_logits (optional) receives the logits of position pos0 + n - 1.
 * Returns that position's greedy token (lowest index on ties), -1 when a
 * logit is not finite, -2 on invalid arguments or a device error (message
 * in error). On a tensor-parallel group every rank makes the same call
 * (the chunks run through the tensor-parallel batched step). The first
 * call allocates the batched step's working buffers (make it before any
 * stream capture). */
int engine_prefill(LLMModel *model, const int *tokens, int n, int pos0, float *last_logits, char *error,
                   size_t error_capacity);

/* Set the keys and values of positions [pos0, pos0 + npos) of layer `layer`
 * directly: seq -1 for the cache engine_forward uses, seq >= 0 for a
 * batched sequence (after engine_batch_open; pos0 must not leave a gap
 * after the sequence's filled positions, and the written positions count
 * as filled). k and v are npos rows of n_kv_heads * head_size floats (all
 * KV heads; a tensor-parallel rank keeps its own), stored as the cache holds
 * them (float, or rounded to half with POCKET_CUDA_KV=f16). This is how a
 * caller restores a saved context, and how the parity tests reach long
 * contexts without decoding them (the reference's CPU engine takes the same
 * rows into its GGUFTransformer state, include/gguf_forward.h:20-31). No
 * counterpart in the reference's engine.h. Returns 1, or 0 with a message. */
int engine_kv_write(LLMModel *model, int seq, int layer, int pos0, int npos, const float *k, const float *v,
                    char *error, size_t error_capacity);

#ifdef __cplusplus
}
#endif

#endif
