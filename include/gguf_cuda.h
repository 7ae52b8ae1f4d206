/*
 * gguf_cuda.h - the fused dequant-matvec of the reference, on the device.
 *
 * GGUFWeight has the layout of the reference's include/gguf_model.h:36-45
 * with one difference of meaning: `data` is a DEVICE pointer to the packed
 * rows (bytes exactly as stored in the GGUF file). Row r starts at
 * data + r * row_bytes.
 *
 * GGML type ids: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K.
 * All calls are asynchronous on `stream` (a cudaStream_t, NULL for the
 * default stream); x, out and data are device pointers. Return 1 on
 * success, 0 on bad arguments or an unsupported type (nothing launched).
 */
#ifndef GGUF_CUDA_H
#define GGUF_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const char *name;     /* optional label */
    const void *data;     /* device pointer to row 0 */
    uint32_t type;        /* GGML type id */
    uint64_t cols;        /* ne0: input length */
    uint64_t rows;        /* ne1: output length */
    uint64_t row_bytes;   /* (cols / block_weights) * block_bytes */
    uint64_t byte_size;   /* rows * row_bytes */
} GGUFWeight;

/*
 * out[r] = sum_c W[r][c] * x[c] for r < rows, read from the packed blocks
 * with no FP32 copy of W. Replaces gguf_matvec, reference
 * include/gguf_model.h:141-145 / src/gguf_model.c:693-771 (same argument
 * meaning; out must not alias x). Agrees with the reference's fast kernels
 * to float32 rounding (relative L2 ~1e-7).
 */
int gguf_cuda_matvec(const GGUFWeight *weight, const float *x, float *out, void *stream);

/*
 * Whether a gguf_cuda_matvec call on the current device has given up on a
 * wait inside its kernel (a weight copy that did not complete in ~2 s)
 * since the last query; read and cleared (synchronises the device). 0: no
 * call's output was affected; 1: at least one call returned with rows it
 * could not compute (their output is invalid); -1: the word cannot be
 * read. Every call starts with a clean abort word, so one such event does
 * not affect later calls. No counterpart in the reference, whose matvec
 * has no device waits.
 */
int gguf_cuda_matvec_error(void);

/*
 * Decode rows [row0, row0 + nrows) to FP32 into out (nrows * cols floats),
 * bit-identical to the reference's gguf_weight_dequantize_row
 * (include/gguf_model.h:112-116, src/gguf_model.c:314-359) and block
 * decoders (src/gguf_quant.c:92-407).
 */
int gguf_cuda_dequantize_rows(const GGUFWeight *weight, uint64_t row0, uint64_t nrows,
                              float *out, void *stream);

/*
 * out[h] = FP32 value of half-precision bit pattern h for all 65536 h,
 * bit-identical to gguf_fp16_to_fp32 (src/gguf_quant.c:6-59), NaN
 * payloads included.
 */
int gguf_cuda_fp16_table(float *out65536, void *stream);

/*
 * Column limit of gguf_cuda_matvec_noalloc: its scratch holds x in integer
 * form for at most this many columns (640 units of 64).
 */
#define GGUF_CUDA_NOALLOC_MAX_COLS 40960

/*
 * gguf_cuda_matvec without any device allocation, ever: the same product,
 * bit for bit, as gguf_cuda_matvec, for callers that must not allocate
 * device memory - a runtime that has reserved all free memory for its own
 * pool, or a latency-critical loop that cannot take cudaMalloc's implicit
 * synchronisation (gguf_cuda_matvec allocates a 4-byte error word on its
 * first call on each device). This entry point has no counterpart in the
 * reference.
 *
 * Scratch: a fixed 184,576-byte array in this library's device code (one
 * per device, created when the device code is loaded): a 256-byte header
 * whose first word is the tile kernel's error word, cleared by every call,
 * then x in integer form, written by a staging kernel and read by every
 * CTA of the tile kernel.
 *
 * - The first call on each device resolves the scratch address with that
 *   device current (cudaGetSymbolAddress, which also loads the device code
 *   when loading is lazy); make that first call before any stream capture.
 * - cols > GGUF_CUDA_NOALLOC_MAX_COLS is rejected (returns 0, message in
 *   `error`).
 * - Calls on one device share the scratch: calls that may overlap in time
 *   (different streams, not ordered by events) race and can return wrong
 *   results. Serialise them, e.g. on one stream.
 * - A wait inside the kernel that gives up (a weight copy that did not
 *   complete in ~2 s) is recorded in the scratch header; read it with
 *   gguf_cuda_matvec_noalloc_error().
 *
 * Returns 1 when the kernels were enqueued on `stream`, 0 otherwise with a
 * message in error[0 .. error_capacity) (may be NULL).
 */
int gguf_cuda_matvec_noalloc(const GGUFWeight *weight, const float *x, float *out, void *stream,
                             char *error, size_t error_capacity);

/*
 * gguf_cuda_matvec_error for gguf_cuda_matvec_noalloc on the current
 * device: read and clear the accumulated error word in the fixed scratch
 * (cudaMemcpyFromSymbol / cudaMemcpyToSymbol, which allocate nothing and
 * synchronise). 0: no call gave up on a wait since the last query; 1: at
 * least one did (its output is invalid); -1: the word cannot be read. No
 * counterpart in the reference.
 */
int gguf_cuda_matvec_noalloc_error(void);

/*
 * Batched counterpart of gguf_cuda_matvec on the tensor cores: for n
 * activation vectors (1 <= n <= 64) that share one pass over the packed
 * weights,
 *     out[b * rows + r] = sum_c W[r][c] * x[b * cols + c],  b < n, r < rows,
 * i.e. gguf_matvec (reference include/gguf_model.h:141-145) applied to each
 * of n vectors. x is n x cols and out is n x rows, row-major, device
 * pointers; out must not overlap x. Q4_K (type 12) and Q5_K (type 13)
 * weights; other types return 0. Every column agrees with gguf_cuda_matvec / the
 * reference's kernel to float32 rounding (the products run on fp16
 * operands that carry x to 22 significant bits, exact products, fp32
 * accumulation). No counterpart in the reference, whose decode runs one
 * sequence at a time.
 *
 * Scratch (staged x, partial sums) is allocated per device on first use
 * and grown on demand; make the first call with the largest n and shape
 * before any stream capture. Calls on one device share the scratch:
 * serialise calls that may overlap in time (e.g. one stream).
 */
int gguf_cuda_matmul(const GGUFWeight *weight, const float *x, int n, float *out, void *stream);

/*
 * The work split gguf_cuda_matmul uses for `rows` rows of `nsb` 256-column
 * super-blocks on `sms` SMs: *ctas CTAs (one per SM at most) and *maxp,
 * the most CTAs that share one 128-row tile. Host-only.
 */
void gguf_cuda_matmul_plan(int rows, int nsb, int sms, int *ctas, int *maxp);

/*
 * The error word of gguf_cuda_matmul on the current device, read and
 * cleared (synchronises the device): 0 when no wait inside the kernel has
 * run out of time since the last read, 1 when one has (that call's output
 * is invalid), -1 when it cannot be read.
 */
int gguf_cuda_matmul_error(void);

#ifdef __cplusplus
}
#endif

#endif
