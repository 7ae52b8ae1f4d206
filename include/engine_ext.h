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
 * device timestamps (ns, %globaltimer, taken by CTA 0) of the last decode
 * step into out and returns how many were written (0 when tracing is off):
 * the step's start, then for each of its 5 * n_layers + 1 phases the time
 * after staging the input vector, after the phase's work and after the
 * grid barrier that ends it. */
int engine_trace(LLMModel *model, unsigned long long *out, int cap);

/* Message of the last device error of this handle ("" if none). */
const char *engine_last_error(const LLMModel *model);

/* Bytes of packed weights resident on the device. */
size_t engine_weight_bytes(const LLMModel *model);

/* Kernel launches one decode step makes: 2 in the default mode (the
 * cooperative step kernel and the one-thread token kernel), one per phase
 * plus one (5 * n_layers + 2) with POCKET_CUDA_PERSISTENT=0 or when the GPU
 * cannot co-schedule the step kernel; 0 for a NULL handle. */
int engine_launches_per_step(const LLMModel *model);

#ifdef __cplusplus
}
#endif

#endif
