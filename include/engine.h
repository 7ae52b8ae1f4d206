/*
 * engine.h - the model interface of the reference engine, served by the
 * B200 decode path.
 *
 * Every declaration matches the reference's include/engine.h:27-90 in name,
 * signature, argument meaning and error behaviour, so callers written for it
 * (the pocket library, benchmarks, the ctypes wrapper) relink unchanged:
 *
 *   LLMModel *m = engine_open(&options, error, sizeof(error));
 *   float *logits = engine_forward(m, token, pos);
 *   engine_close(m);
 *
 * What differs is where the work runs. engine_open() parses the GGUF file,
 * uploads every weight tensor to device memory byte for byte (packed Q4_0 /
 * Q8_0 / Q4_K / Q5_K / Q6_K blocks, no FP32 copies), allocates the FP32 KV
 * cache on the device and captures one decode step as a CUDA graph.
 * engine_forward() replays it; only the logits come back to host memory.
 * Only GGUF files are accepted (the reference's llama2.c FP32 format is not
 * part of this engine). The CUDA device is POCKET_CUDA_DEVICE (default 0)
 * or the one given to engine_open_device() in engine_ext.h.
 *
 * Errors are values: every function returns NULL / 0 / -1 with a message,
 * never prints, exits or aborts. A handle is not thread-safe; several
 * handles may be open at once.
 */
#ifndef ENGINE_H
#define ENGINE_H

#include "tokenizer.h"
#include "transformer.h"

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    LLM_FORMAT_STORIES = 1, /* llama2.c .bin (rejected by this engine) */
    LLM_FORMAT_GGUF = 2     /* GGUF, quantized */
} LLMFormat;

/* include/engine.h:32-49 of the reference. */
typedef struct {
    const char *model_path;     /* required */
    const char *tokenizer_path; /* optional llama2.c tokenizer.bin replacing the GGUF vocabulary */
    int max_context;            /* 0: min(file context, LLM_DEFAULT_MAX_CONTEXT) */
} LLMOptions;

#define LLM_DEFAULT_MAX_CONTEXT 4096

typedef struct LLMModel LLMModel;

/* Replaces engine_open, reference include/engine.h:56-57 / src/engine.c:229-341.
 * NULL on failure with a message in `error`; partial allocations are freed. */
LLMModel *engine_open(const LLMOptions *options, char *error, size_t error_capacity);

/* Replaces engine_close, include/engine.h:60. Safe on NULL. */
void engine_close(LLMModel *model);

/* Replaces engine_forward, include/engine.h:66 / src/engine.c:347-356.
 * One token at position pos (positions in order; pos 0 restarts and
 * overwrites the cache). Returns vocab_size host floats owned by the model,
 * valid until the next call, or NULL for a NULL model, token outside
 * [0, vocab_size) or pos outside [0, seq_len) (the handle stays usable), or
 * after a device error (the handle is then failed). */
float *engine_forward(LLMModel *model, int token, int pos);

/* include/engine.h:69: configuration in use (seq_len is the capped context). */
const Config *engine_config(const LLMModel *model);

/* include/engine.h:72: the context length stored in the file. */
int engine_file_context(const LLMModel *model);

/* include/engine.h:74. */
LLMFormat engine_format(const LLMModel *model);

/* include/engine.h:75: the vocabulary loaded from the GGUF metadata. */
Tokenizer *engine_tokenizer(LLMModel *model);

/* include/engine.h:78: 2 * layers * seq_len * kv_dim * 4 (device bytes). */
size_t engine_kv_cache_bytes(const LLMModel *model);

/* include/engine.h:84: "GGUF, weights Q4_K x135 Q6_K x21 F32 x45". */
const char *engine_description(const LLMModel *model);

/* include/engine.h:90: 1 for EOS (and for a NULL model). */
int engine_is_stop_token(const LLMModel *model, int token);

#ifdef __cplusplus
}
#endif

#endif
