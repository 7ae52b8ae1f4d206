/*
 * tokenizer.h - the vocabulary record returned by engine_tokenizer().
 *
 * Layout-compatible with the reference's include/tokenizer.h:13-48 so that
 * code built against the reference (its tokenizer_encode / tokenizer_decode
 * operate on this record) reads the vocabulary this library loads from the
 * GGUF metadata. Encoding and decoding text are not part of the decode hot
 * path and are not implemented here.
 */
#ifndef WILD_POINTERS_TOKENIZER_H
#define WILD_POINTERS_TOKENIZER_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    char *text;   /* points into Tokenizer.vocab */
    int id;
} TokenizerIndex;

typedef struct {
    char **vocab;                  /* pieces, U+2581 turned into ' ' */
    float *scores;                 /* merge priority; -inf for tokens merges may not build */
    TokenizerIndex *sorted_vocab;  /* vocab sorted by strcmp */
    size_t vocab_size;
    size_t max_token_length;
    unsigned char byte_pieces[512];/* "\x00\0\x01\0..." single-byte strings */
    int bos_id;
    int eos_id;
    int byte_ids[256];             /* token of each raw byte, -1 if none */
    int *special_ids;              /* unknown / control / user-defined tokens */
    size_t n_special;
    int scores_reconstructed;      /* 1 if all scores were equal and were rebuilt */
} Tokenizer;

/* Release the memory a Tokenizer owns. Safe on a zeroed record. */
void tokenizer_free(Tokenizer *tokenizer);

#ifdef __cplusplus
}
#endif

#endif
