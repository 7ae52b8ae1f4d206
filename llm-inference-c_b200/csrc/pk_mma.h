// pk_mma.h - the tcgen05 batched Q4_K / Q5_K / Q6_K matmul (pk_mma.cu) for other device
// code of this library: the same launch as gguf_cuda_matmul, with scratch
// owned by the caller (so that the launch can be captured in a CUDA graph).
#ifndef PK_MMA_H
#define PK_MMA_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// Device scratch of one launch sequence (sized by pk_mm_need; `arrived`
// zeroed once; launches on one stream may share it).
struct PkMmScratch {
    uint8_t *xs, *x2s;
    float *xinv, *ypart;
    unsigned *arrived;
    int *err;        // error word: a wait that ran out of time sets bit 0
    int smem_max;    // from pk_mm_smem_max
};

struct PkMmNeed {
    size_t xs, x2s, xinv, ypart, arrived;  // bytes
};

// 1 if gguf_cuda_matmul takes this weight (Q4_K or Q5_K, 16-byte aligned rows).
int pk_mm_shape_ok(uint32_t type, uint64_t rows, uint64_t cols, uint64_t row_bytes, const void *data);
// The same for a weight inside the engine's arena, where Q6_K is also taken:
// its rows are read in 16-byte aligned windows that may run up to 14 bytes
// past the matrix, which the arena's padding covers (not a caller's buffer).
int pk_mm_arena_ok(uint32_t type, uint64_t rows, uint64_t cols, uint64_t row_bytes, const void *data);
// Scratch bytes for rows x cols and n vectors on `sms` SMs.
void pk_mm_need(int rows, int cols, int n, int sms, PkMmNeed *need);
// Dynamic shared memory the kernel may use on `dev` (sets the attribute
// once; 0 when the device cannot run the kernel). Call outside capture.
int pk_mm_smem_max(int dev);
// y (n x rows) = x (n x cols) W^T: the staging kernel and the matmul kernel
// on `st`. Returns 1 when both were enqueued.
int pk_mm_run(uint32_t type, const uint8_t *w, uint64_t row_bytes, int rows, int cols, const float *x, int n,
              float *y, const PkMmScratch *s, int sms, cudaStream_t st);

// The same in two parts, for several matrices that multiply one x: stage x
// once (pk_mm_stage), then one launch over up to 3 matrices of `cols`
// columns (pk_mm_run_staged; scratch sized by pk_mm_need for their summed
// rows), each with its own output; all of one format.
struct PkMmSeg {
    uint32_t type;  // GGML type id: Q4_K, Q5_K (or, from the arena, Q6_K)
    const uint8_t *w;
    uint64_t row_bytes;
    int rows;
    float *y;  // n x rows
};
int pk_mm_stage(uint32_t type, const float *x, int n, int cols, const PkMmScratch *s, cudaStream_t st);
int pk_mm_run_staged(const PkMmSeg *seg, int nseg, int cols, int n, const PkMmScratch *s, int sms, cudaStream_t st);

#endif
