/*
 * transformer.h - the model configuration record returned by
 * engine_config().
 *
 * Layout-compatible with Config in the reference's include/transformer.h:58-80
 * (seven ints, rope_dim, three floats, in this order), so programs and
 * ctypes bindings written against the reference read it unchanged. The
 * reference's FP32 llama2.c types (Tensor, TransformerWeights, RunState)
 * belong to its CPU path and are not part of this library.
 */
#ifndef TRANSFORMER_H
#define TRANSFORMER_H

typedef struct {
    int dim;          /* embedding width */
    int hidden_dim;   /* SwiGLU hidden width */
    int n_layers;
    int n_heads;      /* query heads */
    int n_kv_heads;   /* key/value heads (GQA when < n_heads) */
    int vocab_size;
    int seq_len;      /* allocated (possibly capped) context */

    int rope_dim;         /* rotated dimensions per head */
    float rope_freq_base; /* RoPE theta */
    float rms_norm_eps;
    float rope_scale;     /* linear RoPE scaling factor, 1 = none */
} Config;

#endif
