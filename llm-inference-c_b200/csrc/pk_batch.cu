// pk_batch.cu - batched decode: one step for up to 64 independent sequences
// that share one pass over the weights. The reference decodes one sequence
// at a time (src/engine.c:137-407 over src/gguf_forward.c); per sequence
// this step computes the same layer loop (gguf_forward.c: RMSNorm, Q/K/V,
// RoPE, KV-cache append, GQA attention, Wo + residual, RMSNorm, SwiGLU,
// down + residual, final norm, logits), so each sequence's logits are
// those of the single-sequence forward up to float rounding.
//
// Work per layer, all on the device:
//   matmuls      Q4_K weights on the tensor cores (pk_mma.cu); every other
//                format on CUDA cores by mv_tile_kernel, which stages the
//                packed rows in shared memory and decodes each weight once
//                per 64-vector tile;
//   elementwise  embedding rows, residual add + RMSNorm (one kernel), RoPE
//                + cache append, attention, SwiGLU, greedy argmax per
//                sequence.
// The launches of one step are captured once per batch size n in a CUDA
// graph (inputs and outputs through fixed pinned buffers).
//
// KV caches: [sequence][layer][position][kv_dim] fp32, as the reference's
// run state (src/transformer.c: key_cache / value_cache) per sequence.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pk_dev.h"
#include "pk_mma.h"
#include "pk_quant.cuh"

namespace pk {
namespace bt {

constexpr int BMAX = 64;            // sequences per step
constexpr int TR = 64, TK = 256;    // mv_tile_kernel: rows per CTA, columns per staged chunk
constexpr int TH = 128;             // columns per decoded half chunk
constexpr int WS = 68;              // row stride of the decoded tile Ws[k][row'] (floats)
constexpr int XP = TH + 4;          // row stride of the x tile Xs[b][k] (floats)
constexpr int MV_SMEM = TH * WS * 4 + BMAX * XP * 4;

// Position of tile row r inside a row of Ws: rows 32..63 shifted by 4 words
// so that the eight 8-row groups read by one warp start on eight different
// 4-bank groups (conflict-free 16-byte loads).
__host__ __device__ constexpr int wpos(int r)
{
    return r + 4 * (r >> 5);
}

__device__ __forceinline__ float block_sum(float v, float *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
    return t;
}

__device__ __forceinline__ float block_max(float v, float *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) t = fmaxf(t, red[w]);
    return t;
}

// Bytes of 256 columns of a row of type T (one K-quant super-block, eight
// Q4_0 / Q8_0 blocks, 256 F16 / F32 values).
template <int T>
__host__ __device__ constexpr int chunk_bytes()
{
    return T == T_Q4_K ? 144 : T == T_Q5_K ? 176 : T == T_Q6_K ? 210 : T == T_Q4_0 ? 144 : T == T_Q8_0 ? 272
         : T == T_F16 ? 512 : 1024;
}

// Halfwords per staged row in shared memory: the chunk's bytes padded to
// an odd number of 4-byte words, so that 32 lanes reading the same offset
// of 32 consecutive rows hit 32 different banks.
template <int T>
__host__ __device__ constexpr int raw_stride()
{
    return 2 * (((chunk_bytes<T>() + 3) / 4) | 1);
}

template <int T>
__host__ __device__ constexpr int mv_smem()
{
    return TR * raw_stride<T>() * 2 + MV_SMEM;
}

// y[b][r] = sum_c W[r][c] x[b][c] (b < n <= 64) on CUDA cores. Per CTA 64
// rows and a range of 256-column chunks (split-K over blockIdx.y when the
// row tiles alone are too few for the SMs). Per chunk the packed bytes of
// the 64 rows are staged in shared memory (rows padded to an odd number of
// words; for formats of at most 32 halfwords per thread and 4-byte aligned
// rows the next chunk loads as words during the current chunk's last FMA
// pass, otherwise with batched 2-byte loads); then, per half of 128
// columns, the x columns of every vector arrive by 16-byte async copies,
// each weight is decoded once from shared memory (bit-exact decoders,
// column-major floats; lanes take consecutive rows), and thread (rg, vg)
// accumulates rows 8rg .. 8rg+7 for vectors 2vg, 2vg+1. One split writes y;
// several write partial sums that mv_reduce_kernel adds in split order. Two
// CTAs per SM (about 82 KB of shared memory for the K-quants).
template <int T>
__global__ void __launch_bounds__(256, 2) mv_tile_kernel(const uint8_t *w, uint64_t rb, int rows, int cols,
                                                         const float *x, int n, float *y, float *part, int cps)
{
    constexpr int CB = chunk_bytes<T>();
    constexpr int HW = TR * (CB / 2);       // halfwords of a staged chunk
    constexpr int RS = raw_stride<T>();      // halfwords per row in Wraw
    constexpr int PER = (HW + 255) / 256;   // per thread
    constexpr int BATCH = PER < 8 ? PER : 8;
    extern __shared__ __align__(16) float smt[];
    float *Ws = smt, *Xs = smt + TH * WS;
    uint16_t *Wraw = reinterpret_cast<uint16_t *>(smt + TH * WS + BMAX * XP);
    const int tid = threadIdx.x, rg = tid & 7, vg = tid >> 3;
    const int row0 = blockIdx.x * TR;
    const int nchunks = (cols + TK - 1) / TK;
    const int c0 = blockIdx.y * cps, c1 = min(nchunks, c0 + cps);
    const bool active = 2 * vg < n;  // warp-uniform (a warp holds vg 4w .. 4w+3)
    const int npad = (n + 1) & ~1;
    // decode: row dr (lanes of a warp take consecutive rows, so the stores
    // into Ws are conflict-free), columns dc0, dc0 + 4, ...
    const int dr = tid & (TR - 1), dc0 = tid >> 6;
    float acc[8][2];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i][0] = acc[i][1] = 0.0f;
    // Packed bytes of chunk ch for the 64 rows, as halfwords e = tid + 256 j
    // (fetch/store in batches). Formats whose chunk takes at most 32
    // halfwords per thread load the next chunk as 4-byte words (fetchw:
    // the 4-byte aligned window of each row's chunk, NW words per row) during
    // the current chunk's last FMA pass, and unpack them into Wraw (storew)
    // after it (PREF, when the rows are 4-byte aligned).
    constexpr bool PREF = PER <= 32;
    constexpr int NW = (CB + 2 + 3) / 4;             // words covering a chunk at a 2-byte offset
    constexpr int PERW = (TR * NW + 255) / 256;      // words per thread
    uint32_t pre[PREF ? PERW : 1];
    auto fetch = [&](int ch, uint16_t *raw, int j0) {
        const uint64_t boff = (uint64_t)ch * CB;
        const int have = (int)min((uint64_t)CB, rb - boff) / 2;  // halfwords of this chunk in a row
#pragma unroll
        for (int j = 0; j < BATCH; j++) {
            const int e = tid + 256 * (j0 + j), r = e / (CB / 2), hw = e - r * (CB / 2);
            raw[j] = (j0 + j < PER && e < HW && row0 + r < rows && hw < have)
                         ? ld_u16(w + (size_t)(row0 + r) * rb + boff + 2 * hw)
                         : (uint16_t)0;
        }
    };
    auto store = [&](const uint16_t *raw, int j0) {
#pragma unroll
        for (int j = 0; j < BATCH; j++) {
            const int e = tid + 256 * (j0 + j), r = e / (CB / 2), hw = e - r * (CB / 2);
            if (j0 + j < PER && e < HW) Wraw[r * RS + hw] = raw[j];
        }
    };
    auto fetchw = [&](int ch) {
        const uint64_t boff = (uint64_t)ch * CB, a = boff & ~(uint64_t)3;
        const uint64_t end = min(boff + (uint64_t)CB, rb);  // the row's bytes end here
#pragma unroll
        for (int j = 0; j < (PREF ? PERW : 1); j++) {
            const int q = tid + 256 * j, r = q / NW, k = q - r * NW;
            const uint64_t at = a + 4 * (uint64_t)k;
            uint32_t v = 0u;
            if (q < TR * NW && row0 + r < rows) {
                const uint8_t *src = w + (size_t)(row0 + r) * rb + at;
                if (at + 4 <= end) {
                    v = *reinterpret_cast<const uint32_t *>(src);
                } else if (at + 2 <= end) {
                    v = ld_u16(src);  // never past the row's last byte
                }
            }
            pre[j] = v;
        }
    };
    auto storew = [&](int ch) {
        const int sh = (int)(((uint64_t)ch * CB) & 3) / 2;  // halfwords before the chunk in word 0
#pragma unroll
        for (int j = 0; j < (PREF ? PERW : 1); j++) {
            const int q = tid + 256 * j, r = q / NW, k = q - r * NW;
            if (q < TR * NW) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const int hw = 2 * k + hh - sh;
                    if (hw >= 0 && hw < CB / 2) Wraw[r * RS + hw] = (uint16_t)(pre[j] >> (16 * hh));
                }
            }
        }
    };
    // 4-byte loads need every row to start on a 4-byte boundary
    const bool pref = PREF && ((rb | (uint64_t)(uintptr_t)w) & 3) == 0;
    if (pref && c0 < c1) fetchw(c0);
    for (int ch = c0; ch < c1; ch++) {
        if (pref) {
            storew(ch);  // Wraw is free: the previous chunk's decode is done
        } else {
            for (int j0 = 0; j0 < PER; j0 += BATCH) {
                uint16_t raw[BATCH];
                fetch(ch, raw, j0);
                store(raw, j0);
            }
        }
        for (int hf = 0; hf < TK / TH; hf++) {
            const int k0 = ch * TK + hf * TH, kc = min(TH, cols - k0);
            if (kc <= 0) break;
            // x columns k0 .. k0+kc of every vector (cols and kc are multiples of 4)
            for (int e = tid; e < npad * (TH / 4); e += 256) {
                const int b = e / (TH / 4), k4 = 4 * (e % (TH / 4));
                float *dst = Xs + b * XP + k4;
                if (b < n && k4 < kc) {
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                                     (uint32_t)__cvta_generic_to_shared(dst)),
                                 "l"(x + (size_t)b * cols + k0 + k4)
                                 : "memory");
                } else {
                    *reinterpret_cast<float4 *>(dst) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            __syncthreads();  // the chunk's packed rows are staged; Ws is free
            {
                const uint8_t *rowp = reinterpret_cast<const uint8_t *>(Wraw + dr * RS);
#pragma unroll 4
                for (int dc = dc0; dc < TH; dc += 4) {
                    Ws[dc * WS + wpos(dr)] = dc < kc ? decode_col(T, rowp, hf * TH + dc) : 0.0f;
                }
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
            __syncthreads();
            // the next chunk's packed bytes load during this chunk's last FMA pass
            if (pref && ch + 1 < c1 && (hf + 1 == TK / TH || k0 + TH >= cols)) fetchw(ch + 1);
            if (active) {
                const float *wk = Ws + wpos(8 * rg);
#pragma unroll 4
                for (int k = 0; k < kc; k++) {
                    const float4 w0 = *reinterpret_cast<const float4 *>(wk + k * WS);
                    const float4 w1 = *reinterpret_cast<const float4 *>(wk + k * WS + 4);
                    const float2 xv = make_float2(Xs[(2 * vg) * XP + k], Xs[(2 * vg + 1) * XP + k]);
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        acc[i][0] = fmaf(wv[i], xv.x, acc[i][0]);
                        acc[i][1] = fmaf(wv[i], xv.y, acc[i][1]);
                    }
                }
            }
            __syncthreads();
        }
    }
    if (!active) return;
    float *out = gridDim.y == 1 ? y : part + (size_t)blockIdx.y * n * rows;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = row0 + 8 * rg + i;
        if (r >= rows) break;
        out[(size_t)(2 * vg) * rows + r] = acc[i][0];
        if (2 * vg + 1 < n) out[(size_t)(2 * vg + 1) * rows + r] = acc[i][1];
    }
}

// y = the splits' partial sums, added in split order.
__global__ void mv_reduce_kernel(const float *part, int splits, int count, float *y)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int k = 0; k < splits; k++) s += part[(size_t)k * count + i];
        y[i] = s;
    }
}

// Split-K of mv_tile_kernel for `rows` x `cols`: chunks per split. With
// two CTAs per SM, the launch takes about waves x cps chunk-steps (waves =
// CTAs / (2 sms), rounded up, since a partly filled last wave costs a whole
// one). The split count that minimises that is taken, except that the
// fewest splits within 5% of the minimum win (each split adds a partial
// sum per output to write and reduce). E.g. 2048 x 5632: 8 splits of 3
// chunks, 256 CTAs in one wave (11 splits of 2 would need a second wave
// for 56 CTAs: 4 chunk-steps instead of 3).
__host__ inline int mv_cps(int rows, int cols, int sms)
{
    const int tiles = (rows + TR - 1) / TR, nchunks = (cols + TK - 1) / TK;
    const long long slots = 2LL * (sms > 0 ? sms : 1);
    long long best = -1;
    for (int cps = 1; cps <= nchunks; cps++) {
        const long long ctas = (long long)tiles * ((nchunks + cps - 1) / cps);
        const long long steps = (ctas + slots - 1) / slots * cps;
        if (best < 0 || steps < best) best = steps;
    }
    // the fewest splits (largest cps) within 5% of the best
    for (int cps = nchunks; cps >= 1; cps--) {
        const long long ctas = (long long)tiles * ((nchunks + cps - 1) / cps);
        const long long steps = (ctas + slots - 1) / slots * cps;
        if (steps * 100 <= best * 105) return cps;
    }
    return 1;
}

// x[b] = embedding row tokens[b] (src/gguf_forward.c: the token's row of
// token_embd, decoded).
__global__ void embed_kernel(const uint8_t *embd, uint64_t rb, int type, const int *io, int dim, float *x)
{
    const int b = blockIdx.x, tok = io[b];
    const uint8_t *row = embd + (size_t)tok * rb;
    for (int c = threadIdx.x; c < dim; c += blockDim.x) x[(size_t)b * dim + c] = decode_col(type, row, c);
}

// out[b] = w * (x[b] / sqrt(mean(x[b]^2) + eps)), as rmsnorm in
// src/gguf_forward.c (the same rounding steps as the single-sequence step);
// with delta != NULL the residual x[b] += delta[b] comes first (and is
// stored). One CTA per sequence.
__global__ void __launch_bounds__(1024) rmsnorm_kernel(float *x, const float *delta, const float *w, int dim,
                                                       float eps, float *out)
{
    __shared__ float red[32];
    float *xb = x + (size_t)blockIdx.x * dim;
    float ss = 0.0f;
    if (delta != nullptr) {
        const float *db = delta + (size_t)blockIdx.x * dim;
        for (int c = threadIdx.x; c < dim; c += blockDim.x) {
            const float v = xb[c] + db[c];
            xb[c] = v;
            ss = fmaf(v, v, ss);
        }
    } else {
        for (int c = threadIdx.x; c < dim; c += blockDim.x) ss = fmaf(xb[c], xb[c], ss);
    }
    const float tot = block_sum(ss, red);
    const float m = __fadd_rn(__fdiv_rn(tot, (float)dim), eps);
    const float sc = __fdiv_rn(1.0f, __fsqrt_rn(m));
    for (int c = threadIdx.x; c < dim; c += blockDim.x)
        out[(size_t)blockIdx.x * dim + c] = __fmul_rn(w[c], __fmul_rn(sc, xb[c]));
}

// RoPE on q and k of sequence b at its position (pairs (2i, 2i + 1) of each
// head, cos/sin from the reference's table), then k and v appended to the
// sequence's cache (src/gguf_forward.c:50-66 and the cache writes; a half
// cache rounds each entry to nearest even).
template <typename KV>
__global__ void rope_cache_kernel(float *q, const float *k, const float *v, const float *rope_cs, int rope_dim,
                                  int hs, int qd, int kvd, const int *io, int bmax, int layer, int L, int seq_len,
                                  KV *kc, KV *vc)
{
    const int b = blockIdx.x;
    const int pos = io[bmax + b], seq = io[2 * bmax + b];
    const float *rope = rope_cs + (size_t)pos * rope_dim;
    float *qb = q + (size_t)b * qd;
    for (int p = threadIdx.x; p < qd / 2; p += blockDim.x) {
        const int d0 = (2 * p) % hs;
        if (d0 < rope_dim) {
            const float c = rope[d0], sn = rope[d0 + 1], v0 = qb[2 * p], v1 = qb[2 * p + 1];
            qb[2 * p] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, sn));
            qb[2 * p + 1] = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, c));
        }
    }
    const size_t row = (((size_t)seq * L + layer) * seq_len + pos) * kvd;
    const float *kb = k + (size_t)b * kvd, *vb = v + (size_t)b * kvd;
    for (int p = threadIdx.x; p < kvd / 2; p += blockDim.x) {
        const int d0 = (2 * p) % hs;
        float v0 = kb[2 * p], v1 = kb[2 * p + 1];
        if (d0 < rope_dim) {
            const float c = rope[d0], sn = rope[d0 + 1];
            const float r0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, sn));
            const float r1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, c));
            v0 = r0;
            v1 = r1;
        }
        kv_store(kc, row + 2 * p, v0);
        kv_store(kc, row + 2 * p + 1, v1);
        kv_store(vc, row + 2 * p, vb[2 * p]);
        kv_store(vc, row + 2 * p + 1, vb[2 * p + 1]);
    }
}

// Attention of query head h of sequence b over positions 0 .. pos
// (grouped-query: KV head h / kv_mul), as in src/gguf_forward.c: scores
// q . k_t * scale, softmax, weighted sum of v_t. One thread per position
// for the scores (16-byte loads of its key row, q from shared memory);
// for the weighted sum thread (g, d4) adds float4 d4 of the values of the
// positions t = g mod G, and the G partial sums are added in order.
// 128 threads; hs a multiple of 4, at most 256.
template <typename KV>
__global__ void __launch_bounds__(128) attention_kernel(const float *q, const KV *kc, const KV *vc,
                                                        const int *io, int bmax, int layer, int L, int seq_len,
                                                        int hs, int qd, int kvd, int kv_mul, float scale, float *out)
{
    extern __shared__ __align__(16) float sc[];  // seq_len scores, then hs query values, then 128 x 4 partials
    __shared__ float red[32];
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int P = io[bmax + b] + 1, seq = io[2 * bmax + b];
    float *qs = sc + ((seq_len + 3) & ~3);
    float4 *part = reinterpret_cast<float4 *>(qs + hs);
    for (int d = tid; d < hs; d += blockDim.x) qs[d] = q[(size_t)b * qd + (size_t)h * hs + d];
    __syncthreads();
    const size_t base = ((size_t)seq * L + layer) * seq_len * kvd + (size_t)(h / kv_mul) * hs;
    const int F4 = hs >> 2;
    const float4 *q4 = reinterpret_cast<const float4 *>(qs);
    float m = -INFINITY;
    for (int t = tid; t < P; t += blockDim.x) {
        const KV *kt = kc + base + (size_t)t * kvd;
        float dot = 0.0f;
        for (int i = 0; i < F4; i++) {
            const float4 kv = kv_load4(kt, 4 * (size_t)i), qv = q4[i];
            dot = fmaf(qv.x, kv.x, dot);
            dot = fmaf(qv.y, kv.y, dot);
            dot = fmaf(qv.z, kv.z, dot);
            dot = fmaf(qv.w, kv.w, dot);
        }
        const float v = dot * scale;
        sc[t] = v;
        m = fmaxf(m, v);
    }
    m = block_max(m, red);
    float s = 0.0f;
    for (int t = tid; t < P; t += blockDim.x) {
        const float e = expf(sc[t] - m);
        sc[t] = e;
        s += e;
    }
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (int t = tid; t < P; t += blockDim.x) sc[t] *= inv;
    __syncthreads();
    const int G = blockDim.x / F4, g = tid / F4, d4 = tid - g * F4;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (g < G) {
        const KV *vb = vc + base + 4 * d4;
#pragma unroll 4
        for (int t = g; t < P; t += G) {
            const float4 vv = kv_load4(vb, (size_t)t * kvd);
            const float pt = sc[t];
            o.x = fmaf(pt, vv.x, o.x);
            o.y = fmaf(pt, vv.y, o.y);
            o.z = fmaf(pt, vv.z, o.z);
            o.w = fmaf(pt, vv.w, o.w);
        }
        part[g * F4 + d4] = o;
    }
    __syncthreads();
    if (tid < F4) {
        float4 r = part[tid];
        for (int k = 1; k < G; k++) {
            const float4 pk = part[k * F4 + tid];
            r.x += pk.x;
            r.y += pk.y;
            r.z += pk.z;
            r.w += pk.w;
        }
        reinterpret_cast<float4 *>(out + (size_t)b * qd + (size_t)h * hs)[tid] = r;
    }
}

// Attention of all H = kv_mul query heads of KV head g for sequence b in
// one CTA, so every key and value row is read once per group rather than
// once per query head. Scores: one thread per position computes the H dot
// products from its key row (16-byte loads); softmax: warp w takes heads
// w, w + 16, ...; weighted sum: thread (tg, d4) reads float4 d4 of the
// value rows t = tg mod G (G = 512 / (hs / 4)) once and adds p_h[t] times
// it for every head h, and the G partials are added in order.
// 512 threads, two CTAs per SM (the loads in flight of two CTAs keep HBM
// busier than longer unrolls in one); H <= 8, H * hs / 4 <= 128.
template <typename KV>
__global__ void __launch_bounds__(512, 2) attention_gqa_kernel(const float *q, const KV *kc, const KV *vc,
                                                            const int *io, int bmax, int layer, int L, int seq_len,
                                                            int hs, int qd, int kvd, int H, float scale, float *out)
{
    extern __shared__ __align__(16) float sg[];  // H * hs queries, H rows of seq_len scores, G x H x hs/4 float4 partials
    const int g = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = io[bmax + b] + 1, seq = io[2 * bmax + b];
    const int sl = (seq_len + 3) & ~3, F4 = hs >> 2;
    float *qs = sg, *sc = sg + H * hs;
    for (int i = tid; i < H * hs; i += blockDim.x) qs[i] = q[(size_t)b * qd + (size_t)g * H * hs + i];
    __syncthreads();
    const size_t base = ((size_t)seq * L + layer) * seq_len * kvd + (size_t)g * hs;
    const float4 *q4 = reinterpret_cast<const float4 *>(qs);
    for (int t = tid; t < P; t += blockDim.x) {
        const KV *kt = kc + base + (size_t)t * kvd;
        float dot[8];
#pragma unroll
        for (int h = 0; h < 8; h++) dot[h] = 0.0f;
#pragma unroll 4  // several key loads in flight per thread
        for (int i = 0; i < F4; i++) {
            const float4 kv = kv_load4(kt, 4 * (size_t)i);
#pragma unroll
            for (int h = 0; h < 8; h++) {
                if (h < H) {
                    const float4 qv = q4[h * F4 + i];
                    dot[h] = fmaf(qv.x, kv.x, dot[h]);
                    dot[h] = fmaf(qv.y, kv.y, dot[h]);
                    dot[h] = fmaf(qv.z, kv.z, dot[h]);
                    dot[h] = fmaf(qv.w, kv.w, dot[h]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 8; h++)
            if (h < H) sc[h * sl + t] = dot[h] * scale;
    }
    __syncthreads();
    for (int h = warp; h < H; h += blockDim.x >> 5) {
        float *sh = sc + h * sl;
        float m = -INFINITY;
        for (int t = lane; t < P; t += 32) m = fmaxf(m, sh[t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        float sum = 0.0f;
        for (int t = lane; t < P; t += 32) {
            const float e = expf(sh[t] - m);
            sh[t] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
        const float inv = 1.0f / sum;
        for (int t = lane; t < P; t += 32) sh[t] *= inv;
    }
    __syncthreads();
    // weighted sum: thread (tg, d4) reads float4 d4 of the value rows
    // t = tg mod G once and adds it into all H heads' sums (p_h[t] from
    // shared memory); the G partials of each (head, d4) are added in order.
    const int G = blockDim.x / F4, tg = tid / F4, d4 = tid - tg * F4;
    float4 *part = reinterpret_cast<float4 *>(sc + H * sl);  // [G][H][F4]
    if (tg < G) {
        const KV *vb = vc + base + 4 * d4;
        float4 o[8];
#pragma unroll
        for (int h = 0; h < 8; h++) o[h] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4  // several value loads in flight per thread
        for (int t = tg; t < P; t += G) {
            const float4 vv = kv_load4(vb, (size_t)t * kvd);
#pragma unroll
            for (int h = 0; h < 8; h++) {
                if (h < H) {
                    const float pt = sc[h * sl + t];
                    o[h].x = fmaf(pt, vv.x, o[h].x);
                    o[h].y = fmaf(pt, vv.y, o[h].y);
                    o[h].z = fmaf(pt, vv.z, o[h].z);
                    o[h].w = fmaf(pt, vv.w, o[h].w);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 8; h++)
            if (h < H) part[((size_t)tg * H + h) * F4 + d4] = o[h];
    }
    __syncthreads();
    if (tid < H * F4) {
        const int hh = tid / F4, dd = tid - hh * F4;
        float4 r = part[(size_t)hh * F4 + dd];
        for (int k = 1; k < G; k++) {
            const float4 pk = part[((size_t)k * H + hh) * F4 + dd];
            r.x += pk.x;
            r.y += pk.y;
            r.z += pk.z;
            r.w += pk.w;
        }
        reinterpret_cast<float4 *>(out + (size_t)b * qd + ((size_t)g * H + hh) * hs)[dd] = r;
    }
}

// ------------------------------------------------------------------ //
// Tensor parallel exchanges of the batched step                      //
// ------------------------------------------------------------------ //
//
// Every rank's exchange region holds [2 slots][world][len] 64-bit words
// (tag << 32 | payload). Exchange t (tags are consecutive over all of a
// handle's exchanges; 0 never appears) uses slot t & 1: each rank writes
// its part into part `rank` of that slot on every rank (NVLink stores) and
// then polls its own copy of the other parts until they carry tag t. A
// rank writes slot s again two exchanges later, only after it has read the
// exchange between them, which its peers published after finishing their
// reads of slot s: no word is overwritten before it is read. Every poll is
// bounded and records a timeout in the error word.

constexpr long long TP_WAIT_LIMIT_CYCLES = 20000000000LL;  // ~10 s: a peer may start its step later
constexpr int TP_ERR_TIMEOUT = 2;

struct TpX {
    uint64_t *peer[PKD_TP_MAX];  // each rank's exchange region (slot 0, part 0)
    uint64_t len;                // words per part
    int rank, world;
};

__device__ __forceinline__ void tp_st(uint64_t *p, uint32_t payload, uint32_t tag)
{
    const uint64_t w = ((uint64_t)tag << 32) | payload;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// The payload of the word at p once it carries `tag` (0 after a timeout).
__device__ __forceinline__ uint32_t tp_ld(const uint64_t *p, uint32_t tag, int *err)
{
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
    const long long t0 = clock64();
    for (;;) {
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
        if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
        if ((*(volatile int *)err & TP_ERR_TIMEOUT) || clock64() - t0 > TP_WAIT_LIMIT_CYCLES) {
            atomicOr(err, TP_ERR_TIMEOUT);
            return 0u;
        }
    }
}

// Publish len floats of src as this rank's part of exchange tag0 + idx.
__global__ void tp_push_kernel(TpX x, const float *src, int len, const int *tag0, int idx)
{
    const uint32_t tag = 1u + (uint32_t)tag0[0] + (uint32_t)idx;
    const size_t off = ((size_t)(tag & 1u) * x.world + x.rank) * x.len;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < len; i += gridDim.x * blockDim.x) {
        const uint32_t v = __float_as_uint(src[i]);
        for (int q = 0; q < x.world; q++) tp_st(x.peer[q] + off + i, v, tag);
    }
}

// out[i] = the sum of the ranks' parts in rank order (the all-reduce).
__global__ void tp_sum_kernel(TpX x, float *out, int len, const int *tag0, int idx, int *err)
{
    const uint32_t tag = 1u + (uint32_t)tag0[0] + (uint32_t)idx;
    const uint64_t *mine = x.peer[x.rank] + (size_t)(tag & 1u) * x.world * x.len;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < len; i += gridDim.x * blockDim.x) {
        float s = __uint_as_float(tp_ld(mine + i, tag, err));
        for (int q = 1; q < x.world; q++) s = __fadd_rn(s, __uint_as_float(tp_ld(mine + (size_t)q * x.len + i, tag, err)));
        out[i] = s;
    }
}

// The ranks' logits slices (rank q: n rows of voc[q] floats from column
// voc0[q]) assembled into out[n][vocab].
__global__ void tp_gather_kernel(TpX x, float *out, int n, int vocab, const int *tag0, int idx, int *err)
{
    const uint32_t tag = 1u + (uint32_t)tag0[0] + (uint32_t)idx;
    const uint64_t *mine = x.peer[x.rank] + (size_t)(tag & 1u) * x.world * x.len;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * vocab; i += gridDim.x * blockDim.x) {
        const int b = i / vocab, c = i - b * vocab;
        int q = 0;
        while (q + 1 < x.world && c >= (int)((long long)vocab * (q + 1) / x.world)) q++;
        const int v0 = (int)((long long)vocab * q / x.world), vq = (int)((long long)vocab * (q + 1) / x.world) - v0;
        out[i] = __uint_as_float(tp_ld(mine + (size_t)q * x.len + (size_t)b * vq + (c - v0), tag, err));
    }
}

// Sequence b's greedy token over the ranks' vocabulary slices: the rank's
// largest logit and its lowest index on ties (src/sampler.c:39-52), as an
// ordered key, published to every rank; -1 from any rank that saw a
// non-finite logit.
__global__ void __launch_bounds__(1024) tp_argmax_push_kernel(TpX x, const float *logits, int voc, int voc0,
                                                              const int *tag0, int idx)
{
    __shared__ unsigned long long best_w[32];
    __shared__ int bad_w[32];
    const int b = blockIdx.x, tid = threadIdx.x;
    unsigned long long best = 0ull;
    int bad = 0;
    for (int j = tid; j < voc; j += blockDim.x) {
        const float v = logits[(size_t)b * voc + j];
        if (!isfinite(v)) bad = 1;
        const uint32_t u = __float_as_uint(v);
        const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        const unsigned long long k = ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)(voc0 + j));
        if (k > best) best = k;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        if (ob > best) best = ob;
        bad |= __shfl_xor_sync(0xFFFFFFFFu, bad, o);
    }
    if ((tid & 31) == 0) {
        best_w[tid >> 5] = best;
        bad_w[tid >> 5] = bad;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) {
            if (best_w[w] > best) best = best_w[w];
            bad |= bad_w[w];
        }
        const uint32_t tag = 1u + (uint32_t)tag0[0] + (uint32_t)idx;
        const size_t off = ((size_t)(tag & 1u) * x.world + x.rank) * x.len + (size_t)b * 3;
        for (int q = 0; q < x.world; q++) {
            tp_st(x.peer[q] + off, (uint32_t)(best >> 32), tag);
            tp_st(x.peer[q] + off + 1, (uint32_t)best, tag);
            tp_st(x.peer[q] + off + 2, (uint32_t)bad, tag);
        }
    }
}

__global__ void tp_argmax_kernel(TpX x, int n, int *next, const int *tag0, int idx, int *err)
{
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    const uint32_t tag = 1u + (uint32_t)tag0[0] + (uint32_t)idx;
    const uint64_t *mine = x.peer[x.rank] + (size_t)(tag & 1u) * x.world * x.len;
    unsigned long long best = 0ull;
    bool bad = false;
    for (int q = 0; q < x.world; q++) {
        const uint64_t *w = mine + (size_t)q * x.len + (size_t)b * 3;
        const unsigned long long k = ((unsigned long long)tp_ld(w, tag, err) << 32) | tp_ld(w + 1, tag, err);
        if (k > best) best = k;
        if (tp_ld(w + 2, tag, err) != 0u) bad = true;
    }
    next[b] = (bad || best == 0ull) ? -1 : (int)(0xFFFFFFFFu - (uint32_t)best);
}

// The next step's tags start after this step's `count` exchanges.
__global__ void tp_advance_kernel(int *tag0, int count)
{
    tag0[0] += count;
}

// g = silu(g) * u, the reference's rounding steps (src/gguf_forward.c).
__global__ void swiglu_kernel(float *g, const float *u, int count)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const float v = g[i];
        g[i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u[i]);
    }
}

// Greedy token of sequence b: the largest logit, the lowest index on ties
// (src/sampler.c:39-52); -1 when a logit is not finite.
__global__ void __launch_bounds__(1024) argmax_kernel(const float *logits, int vocab, int *next)
{
    __shared__ float bv[32];
    __shared__ int bi[32], bad[32];
    const float *l = logits + (size_t)blockIdx.x * vocab;
    float best = -INFINITY;
    int idx = 0x7FFFFFFF, nonfinite = 0;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float v = l[i];
        if (!isfinite(v)) nonfinite = 1;
        else if (v > best || (v == best && i < idx)) {
            best = v;
            idx = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
        nonfinite |= __shfl_xor_sync(0xFFFFFFFFu, nonfinite, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        bv[warp] = best;
        bi[warp] = idx;
        bad[warp] = nonfinite;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) {
            nonfinite |= bad[w];
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        }
        next[blockIdx.x] = nonfinite ? -1 : idx;
    }
}

}  // namespace bt
}  // namespace pk

using namespace pk;

struct PkbCtx {
    int device, sms, max_seqs;
    cudaStream_t st;
    PkdModel m;  // tensor tables owned by the PkdCtx
    const uint8_t *arena;
    const float *norms, *rope_cs;
    void *kc, *vc;                                            // [max_seqs][L][seq_len][kvd], float or half
    float *x, *xn, *q, *k, *v, *att, *tmp, *g, *u, *logits;  // [64][width]
    float *part;                                              // split-K partial sums of mv_tile_kernel
    int *io_d, *io_h;  // [tokens 64][pos 64][seq 64][next 64][error word]
    PkMmScratch mm;
    cudaGraph_t graph[2][bt::BMAX + 1];  // per batch size; [1]: with the logits gathered (tensor parallel)
    cudaGraphExec_t exec[2][bt::BMAX + 1];
    // tensor parallel (world > 1): the exchanges of the step, the device
    // counter their tags start from, and the assembled logits
    int world;
    bt::TpX tpx;
    int *tag0;
    float *logits_full;
    int gqa_smem;  // dynamic shared memory of attention_gqa_kernel (0: per-head attention instead)
    int kv_alias;  // kc / vc belong to the decode step (pkb_create_prefill): not freed here
    cudaStream_t side;             // tile-kernel matrices that run beside a tensor-core launch
    cudaEvent_t ev_fork, ev_join;  //   (forked from and joined to st inside the captured step)
    char msg[256];
};

static int bfail(PkbCtx *b, cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return 0;
    snprintf(b->msg, sizeof(b->msg), "CUDA %s failed: %s", what, cudaGetErrorString(e));
    return 1;
}

extern "C" int pkb_kv_write(PkbCtx *b, int seq, int layer, int pos0, int npos, const float *k, const float *v,
                            char *err, size_t cap)
{
    if (b == NULL || k == NULL || v == NULL) return 0;
    const PkdModel &m = b->m;
    if (seq < 0 || seq >= b->max_seqs || layer < 0 || layer >= m.n_layers || pos0 < 0 || npos < 0 ||
        pos0 > m.seq_len - npos) {
        if (err && cap) snprintf(err, cap, "KV write outside the cache.");
        return 0;
    }
    cudaSetDevice(b->device);
    const size_t kvd = (size_t)m.head_size * (size_t)m.n_kv_heads;
    const size_t off = (((size_t)seq * m.n_layers + layer) * (size_t)m.seq_len + (size_t)pos0) * kvd;
    const size_t n = (size_t)npos * kvd;
    cudaError_t e = pk::kv_upload(b->kc, m.kv_half, off, k, n, b->st);
    if (e == cudaSuccess) e = pk::kv_upload(b->vc, m.kv_half, off, v, n, b->st);
    if (e != cudaSuccess) {
        if (err && cap) snprintf(err, cap, "CUDA KV write failed: %s", cudaGetErrorString(e));
        return 0;
    }
    return 1;
}

// y (n x rows) = x (n x cols) W^T for one weight tensor.
// tc: the tensor-core launch may be used (not beside another launch that
// shares its staging scratch).
static int bmatmul(PkbCtx *b, const PkdTensor &t, const float *x, int n, float *y, cudaStream_t st = nullptr,
                   bool tc = true)
{
    if (st == nullptr) st = b->st;
    const uint8_t *w = b->arena + t.offset;
    const int rows = (int)t.rows, cols = (int)t.cols;
    if (tc && pk_mm_arena_ok(t.type, t.rows, t.cols, t.row_bytes, w))
        return pk_mm_run(t.type, w, t.row_bytes, rows, cols, x, n, y, &b->mm, b->sms, st);
    const int cps = bt::mv_cps(rows, cols, b->sms), nchunks = (cols + bt::TK - 1) / bt::TK;
    const int splits = (nchunks + cps - 1) / cps;
    const dim3 grid((rows + bt::TR - 1) / bt::TR, splits);
    switch (t.type) {
#define PKB_CASE(T)                                                                                           \
    case T:                                                                                                   \
        bt::mv_tile_kernel<T><<<grid, 256, bt::mv_smem<T>(), st>>>(w, t.row_bytes, rows, cols, x, n, y,       \
                                                                   b->part, cps);                             \
        break;
        PKB_CASE(T_F32)
        PKB_CASE(T_F16)
        PKB_CASE(T_Q4_0)
        PKB_CASE(T_Q8_0)
        PKB_CASE(T_Q4_K)
        PKB_CASE(T_Q5_K)
        PKB_CASE(T_Q6_K)
#undef PKB_CASE
    default:
        return 0;
    }
    if (splits > 1) {
        const int count = n * rows;
        bt::mv_reduce_kernel<<<(count + 255) / 256, 256, 0, st>>>(b->part, splits, count, y);
    }
    return cudaGetLastError() == cudaSuccess;
}

// y_i = x W_i^T for weights that multiply the same x: the ones of the first
// tensor-core format (Q4_K, Q5_K or Q6_K) in one tensor-core launch (x
// staged once), the others (a second format included) on the tile kernel. When
// both kinds are present the tile-kernel ones run on a side stream, forked
// before and joined after the tensor-core launch, so that they use the SMs
// the tensor-core grid leaves idle (e.g. the Q6_K attn_v of an even layer
// beside the Q and K launch of 32 CTAs). Their outputs and the tile
// kernel's split-K partials are not touched by the tensor-core launch.
static int bmatmul_group(PkbCtx *b, const PkdTensor *const *ts, float *const *ys, int cnt, const float *x, int n)
{
    PkMmSeg seg[3];
    int ns = 0, tiles = 0;
    uint32_t tc_type = 0;  // the tensor-core launch takes the first tensor-core format's matrices
    auto in_launch = [&](const PkdTensor &t) {
        return pk_mm_arena_ok(t.type, t.rows, t.cols, t.row_bytes, b->arena + t.offset) && t.type == tc_type;
    };
    for (int i = 0; i < cnt; i++) {
        const PkdTensor &t = *ts[i];
        if (tc_type == 0 && pk_mm_arena_ok(t.type, t.rows, t.cols, t.row_bytes, b->arena + t.offset)) tc_type = t.type;
    }
    for (int i = 0; i < cnt; i++) {
        if (in_launch(*ts[i])) {
            ns++;
        } else {
            tiles++;
        }
    }
    const bool fork = ns > 0 && tiles > 0;
    if (fork && (bfail(b, cudaEventRecord(b->ev_fork, b->st), "event") ||
                 bfail(b, cudaStreamWaitEvent(b->side, b->ev_fork, 0), "event"))) {
        return 0;
    }
    ns = 0;
    for (int i = 0; i < cnt; i++) {
        const PkdTensor &t = *ts[i];
        const uint8_t *w = b->arena + t.offset;
        if (in_launch(t)) {
            seg[ns].type = t.type;
            seg[ns].w = w;
            seg[ns].row_bytes = t.row_bytes;
            seg[ns].rows = (int)t.rows;
            seg[ns].y = ys[i];
            ns++;
        } else if (!bmatmul(b, t, x, n, ys[i], fork ? b->side : b->st, false)) {
            return 0;
        }
    }
    if (ns == 0) return 1;
    const int cols = (int)ts[0]->cols;
    if (!pk_mm_stage(tc_type, x, n, cols, &b->mm, b->st) ||
        !pk_mm_run_staged(seg, ns, cols, n, &b->mm, b->sms, b->st)) {
        return 0;
    }
    return !fork || (!bfail(b, cudaEventRecord(b->ev_join, b->side), "event") &&
                     !bfail(b, cudaStreamWaitEvent(b->st, b->ev_join, 0), "event"));
}

// Layer l's KV append (after RoPE) and attention for the n rows of a step,
// over a cache of KV entries (float or half).
template <typename KV>
static void attend(PkbCtx *b, int l, int n, size_t att_smem, KV *kc, KV *vc)
{
    const PkdModel &m = b->m;
    const int hs = m.head_size, qd = m.n_heads * hs, kvd = m.n_kv_heads * hs, L = m.n_layers, B = bt::BMAX;
    cudaStream_t st = b->st;
    bt::rope_cache_kernel<KV><<<n, 256, 0, st>>>(b->q, b->k, b->v, b->rope_cs, m.rope_dim, hs, qd, kvd, b->io_d, B,
                                                 l, L, m.seq_len, kc, vc);
    if (b->gqa_smem > 0) {
        bt::attention_gqa_kernel<KV><<<dim3(m.n_kv_heads, n), 512, b->gqa_smem, st>>>(
            b->q, kc, vc, b->io_d, B, l, L, m.seq_len, hs, qd, kvd, m.n_heads / m.n_kv_heads, m.att_scale, b->att);
    } else {
        bt::attention_kernel<KV><<<dim3(m.n_heads, n), 128, att_smem, st>>>(
            b->q, kc, vc, b->io_d, B, l, L, m.seq_len, hs, qd, kvd, m.n_heads / m.n_kv_heads, m.att_scale, b->att);
    }
}

// The launches of one step for n sequences (inputs already in io_d).
// This rank's part of an all-reduce (sum) of len floats at y, in place.
static void tp_allreduce(PkbCtx *b, float *y, int len, int &idx)
{
    const int grid = (len + 255) / 256 < 2 * b->sms ? (len + 255) / 256 : 2 * b->sms;
    bt::tp_push_kernel<<<grid, 256, 0, b->st>>>(b->tpx, y, len, b->tag0, idx);
    bt::tp_sum_kernel<<<grid, 256, 0, b->st>>>(b->tpx, y, len, b->tag0, idx, b->mm.err);
    idx++;
}

static int enqueue_step(PkbCtx *b, int n, int with_logits)
{
    const PkdModel &m = b->m;
    const int dim = m.dim, hs = m.head_size, hid = m.hidden_dim;
    const int L = m.n_layers, B = bt::BMAX;
    cudaStream_t st = b->st;
    const int ew = (n * (hid > dim ? hid : dim) + 255) / 256;
    bt::embed_kernel<<<n, 256, 0, st>>>(b->arena + m.embd.offset, m.embd.row_bytes, (int)m.embd.type, b->io_d, dim,
                                        b->x);
    const size_t att_smem = (((size_t)m.seq_len + 3) / 4 * 4 + hs + 128 * 4) * 4;
    int tix = 0;  // this step's tensor-parallel exchanges so far
    for (int l = 0; l < L; l++) {
        if (l == 0)  // later layers: the residual add and this norm at the end of the previous layer
            bt::rmsnorm_kernel<<<n, 1024, 0, st>>>(b->x, nullptr, b->norms, dim, m.rms_eps, b->xn);
        const PkdTensor *qkv[3] = {&m.wq[l], &m.wk[l], &m.wv[l]};
        float *const qkv_y[3] = {b->q, b->k, b->v};
        if (!bmatmul_group(b, qkv, qkv_y, 3, b->xn, n)) return 0;
        if (m.kv_half) {
            attend(b, l, n, att_smem, static_cast<__half *>(b->kc), static_cast<__half *>(b->vc));
        } else {
            attend(b, l, n, att_smem, static_cast<float *>(b->kc), static_cast<float *>(b->vc));
        }
        if (!bmatmul(b, m.wo[l], b->att, n, b->tmp)) return 0;
        if (b->world > 1) tp_allreduce(b, b->tmp, n * dim, tix);  // the heads' partial sums
        bt::rmsnorm_kernel<<<n, 1024, 0, st>>>(b->x, b->tmp, b->norms + (size_t)(2 * l + 1) * dim, dim, m.rms_eps,
                                               b->xn);
        const PkdTensor *gu[2] = {&m.gate[l], &m.up[l]};
        float *const gu_y[2] = {b->g, b->u};
        if (!bmatmul_group(b, gu, gu_y, 2, b->xn, n)) return 0;
        bt::swiglu_kernel<<<ew, 256, 0, st>>>(b->g, b->u, n * hid);
        if (!bmatmul(b, m.down[l], b->g, n, b->tmp)) return 0;
        if (b->world > 1) tp_allreduce(b, b->tmp, n * dim, tix);  // the hidden slices' partial sums
        // x += down, then the next layer's attention norm (the output norm after the last)
        bt::rmsnorm_kernel<<<n, 1024, 0, st>>>(b->x, b->tmp, b->norms + (size_t)(2 * (l + 1)) * dim, dim,
                                               m.rms_eps, b->xn);
    }
    if (!bmatmul(b, m.output, b->xn, n, b->logits)) return 0;
    if (b->world > 1) {
        // the vocabulary rows of this rank: local keys, the best over ranks
        const int voc = (int)m.output.rows, voc0 = m.tp.voc0;
        bt::tp_argmax_push_kernel<<<n, 1024, 0, st>>>(b->tpx, b->logits, voc, voc0, b->tag0, tix);
        bt::tp_argmax_kernel<<<1, 64, 0, st>>>(b->tpx, n, b->io_d + 3 * B, b->tag0, tix, b->mm.err);
        tix++;
        if (with_logits) {
            const int len = n * voc, grid = (len + 255) / 256 < 2 * b->sms ? (len + 255) / 256 : 2 * b->sms;
            bt::tp_push_kernel<<<grid, 256, 0, st>>>(b->tpx, b->logits, len, b->tag0, tix);
            const int all = n * m.vocab_size;
            bt::tp_gather_kernel<<<(all + 255) / 256 < 4 * b->sms ? (all + 255) / 256 : 4 * b->sms, 256, 0, st>>>(
                b->tpx, b->logits_full, n, m.vocab_size, b->tag0, tix, b->mm.err);
            tix++;
        }
        bt::tp_advance_kernel<<<1, 1, 0, st>>>(b->tag0, tix);
    } else {
        bt::argmax_kernel<<<n, 1024, 0, st>>>(b->logits, m.vocab_size, b->io_d + 3 * B);
    }
    // the greedy tokens and the matmul error word come back with the step
    cudaMemcpyAsync(b->io_d + 4 * B, b->mm.err, sizeof(int), cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(b->io_h + 3 * B, b->io_d + 3 * B, (B + 1) * sizeof(int), cudaMemcpyDeviceToHost, st);
    return cudaGetLastError() == cudaSuccess;
}

static PkbCtx *pkb_create_ex(PkdCtx *ctx, int max_seqs, int alias, char *err, size_t cap);

extern "C" PkbCtx *pkb_create(PkdCtx *ctx, int max_seqs, char *err, size_t cap)
{
    return pkb_create_ex(ctx, max_seqs, 0, err, cap);
}

extern "C" PkbCtx *pkb_create_prefill(PkdCtx *ctx, char *err, size_t cap)
{
    return pkb_create_ex(ctx, 1, 1, err, cap);
}

static PkbCtx *pkb_create_ex(PkdCtx *ctx, int max_seqs, int alias, char *err, size_t cap)
{
    PkdView v;
    if (!pkd_view(ctx, &v)) {
        if (err && cap) snprintf(err, cap, "Batched decode needs a built model (tensor parallel: after the connect).");
        return NULL;
    }
    if (max_seqs < 1 || max_seqs > bt::BMAX) {
        if (err && cap) snprintf(err, cap, "Batched decode takes 1 to %d sequences.", bt::BMAX);
        return NULL;
    }
    const PkdModel &m = *v.model;
    if ((m.head_size & 3) || m.head_size > 256 || m.rope_dim > m.head_size || (m.rope_dim & 1)) {
        if (err && cap) snprintf(err, cap, "Unsupported model shape for batched decode.");
        return NULL;
    }
    PkbCtx *b = (PkbCtx *)calloc(1, sizeof(PkbCtx));
    if (b == NULL) {
        if (err && cap) snprintf(err, cap, "Out of memory.");
        return NULL;
    }
    b->device = v.device;
    b->st = (cudaStream_t)v.stream;
    cudaSetDevice(b->device);
    if (bfail(b, cudaStreamCreateWithFlags(&b->side, cudaStreamNonBlocking), "cudaStreamCreate") ||
        bfail(b, cudaEventCreateWithFlags(&b->ev_fork, cudaEventDisableTiming), "cudaEventCreate") ||
        bfail(b, cudaEventCreateWithFlags(&b->ev_join, cudaEventDisableTiming), "cudaEventCreate")) {
        if (err && cap) snprintf(err, cap, "%s", b->msg);
        pkb_destroy(b);
        return NULL;
    }
    b->m = m;
    b->arena = v.arena;
    b->norms = v.norms;
    b->rope_cs = v.rope_cs;
    b->max_seqs = max_seqs;
    b->world = v.world;
    if (v.world > 1) {
        b->tpx.rank = v.rank;
        b->tpx.world = v.world;
        b->tpx.len = v.bx_len;
        for (int q = 0; q < v.world; q++) b->tpx.peer[q] = v.peers[q] + v.bx;
        if (bfail(b, cudaMalloc(&b->tag0, 16), "cudaMalloc") || bfail(b, cudaMemset(b->tag0, 0, 16), "cudaMemset") ||
            bfail(b, cudaMalloc(&b->logits_full, (size_t)bt::BMAX * m.vocab_size * 4), "cudaMalloc")) {
            if (err && cap) snprintf(err, cap, "%s", b->msg);
            pkb_destroy(b);
            return NULL;
        }
    }
    cudaSetDevice(b->device);
    cudaDeviceGetAttribute(&b->sms, cudaDevAttrMultiProcessorCount, b->device);
    const int B = bt::BMAX, dim = m.dim, hs = m.head_size, qd = m.n_heads * hs, kvd = m.n_kv_heads * hs;
    const size_t cache = (size_t)max_seqs * m.n_layers * m.seq_len * kvd * (m.kv_half ? 2 : 4);  // bytes
    // matmul scratch: the largest need over the model's Q4_K launches at
    // n = 64 (Q/K/V and gate/up each one launch of their Q4_K matrices)
    PkMmNeed mx = {0, 0, 0, 0, 0};
    const PkdTensor *lists[7] = {m.wq, m.wk, m.wv, m.wo, m.gate, m.up, m.down};
    auto consider = [&](int rows, int cols) {
        if (rows == 0) return;
        PkMmNeed nd;
        pk_mm_need(rows, cols, B, b->sms, &nd);
        if (nd.xs > mx.xs) mx.xs = nd.xs;
        if (nd.x2s > mx.x2s) mx.x2s = nd.x2s;
        if (nd.xinv > mx.xinv) mx.xinv = nd.xinv;
        if (nd.ypart > mx.ypart) mx.ypart = nd.ypart;
        if (nd.arrived > mx.arrived) mx.arrived = nd.arrived;
    };
    auto q4k_rows = [&](const PkdTensor &t) -> int {
        return pk_mm_arena_ok(t.type, t.rows, t.cols, t.row_bytes, v.arena + t.offset) ? (int)t.rows : 0;
    };
    for (int l = 0; l < m.n_layers; l++) {
        consider(q4k_rows(m.wq[l]) + q4k_rows(m.wk[l]) + q4k_rows(m.wv[l]), m.dim);
        consider(q4k_rows(m.wo[l]), (int)m.wo[l].cols);
        consider(q4k_rows(m.gate[l]) + q4k_rows(m.up[l]), m.dim);
        consider(q4k_rows(m.down[l]), (int)m.down[l].cols);
    }
    consider(q4k_rows(m.output), m.dim);
    size_t part_max = 16;
    for (int j = 0; j <= 7 * m.n_layers; j++) {
        const PkdTensor &t = j == 7 * m.n_layers ? m.output : lists[j / m.n_layers][j % m.n_layers];
        const int cps = bt::mv_cps((int)t.rows, (int)t.cols, b->sms);
        const int splits = ((int)((t.cols + bt::TK - 1) / bt::TK) + cps - 1) / cps;
        if (splits > 1 && (size_t)splits * B * t.rows * 4 > part_max) part_max = (size_t)splits * B * t.rows * 4;
    }
    b->mm.smem_max = pk_mm_smem_max(b->device);
    int ok = b->mm.smem_max > 0 || mx.xs == 0;
    if (!ok) snprintf(b->msg, sizeof(b->msg), "The tensor-core matmul cannot run on this device.");
    if (alias) {
        b->kc = v.kc;
        b->vc = v.vc;
        b->kv_alias = 1;
    }
    ok = ok && (alias || (!bfail(b, cudaMalloc(&b->kc, cache), "cudaMalloc(batched KV cache)") &&
                          !bfail(b, cudaMalloc(&b->vc, cache), "cudaMalloc(batched KV cache)"))) &&
         !bfail(b, cudaMalloc(&b->x, (size_t)B * dim * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->xn, (size_t)B * dim * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->tmp, (size_t)B * dim * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->q, (size_t)B * qd * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->att, (size_t)B * qd * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->k, (size_t)B * kvd * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->v, (size_t)B * kvd * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->g, (size_t)B * m.hidden_dim * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->u, (size_t)B * m.hidden_dim * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->logits, (size_t)B * m.vocab_size * 4), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->part, part_max), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->io_d, (size_t)(5 * B) * 4), "cudaMalloc") &&
         !bfail(b, cudaMallocHost(&b->io_h, (size_t)(5 * B) * 4), "cudaMallocHost") &&
         !bfail(b, cudaMalloc(&b->mm.xs, mx.xs + 16), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->mm.x2s, mx.x2s + 16), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->mm.xinv, mx.xinv + 16), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->mm.ypart, mx.ypart + 16), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->mm.arrived, mx.arrived + 16), "cudaMalloc") &&
         !bfail(b, cudaMalloc(&b->mm.err, 16), "cudaMalloc") &&
         !bfail(b, cudaMemsetAsync(b->mm.arrived, 0, mx.arrived + 16, b->st), "cudaMemset") &&
         !bfail(b, cudaMemsetAsync(b->mm.err, 0, 16, b->st), "cudaMemset") &&
         (alias || (!bfail(b, cudaMemsetAsync(b->kc, 0, cache, b->st), "cudaMemset") &&
                    !bfail(b, cudaMemsetAsync(b->vc, 0, cache, b->st), "cudaMemset")));
#define PKB_ATTR(T)                                                                                           \
    ok = ok && !bfail(b, cudaFuncSetAttribute(bt::mv_tile_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                              bt::mv_smem<T>()),                                              \
                      "cudaFuncSetAttribute");
    PKB_ATTR(T_F32)
    PKB_ATTR(T_F16)
    PKB_ATTR(T_Q4_0)
    PKB_ATTR(T_Q8_0)
    PKB_ATTR(T_Q4_K)
    PKB_ATTR(T_Q5_K)
    PKB_ATTR(T_Q6_K)
#undef PKB_ATTR
    const size_t att_smem = (((size_t)m.seq_len + 3) / 4 * 4 + hs + 128 * 4) * 4;
    if (ok && att_smem > 48 * 1024)
        ok = !bfail(b, cudaFuncSetAttribute(bt::attention_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)att_smem),
                    "cudaFuncSetAttribute") &&
             !bfail(b, cudaFuncSetAttribute(bt::attention_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)att_smem),
                    "cudaFuncSetAttribute");
    // grouped attention when a CTA can hold the group's queries and scores
    // and the group fills at least half of its threads
    {
        const int H = m.n_heads / m.n_kv_heads;
        const size_t gs = ((size_t)H * hs + (size_t)H * ((m.seq_len + 3) / 4 * 4)) * 4 + (size_t)512 * H * 16;
        if (ok && H >= 2 && H <= 8 && H * (hs / 4) >= 64 && H * (hs / 4) <= 128 && gs <= 200 * 1024) {
            ok = !bfail(b, cudaFuncSetAttribute(bt::attention_gqa_kernel<float>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gs),
                        "cudaFuncSetAttribute") &&
                 !bfail(b, cudaFuncSetAttribute(bt::attention_gqa_kernel<__half>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gs),
                        "cudaFuncSetAttribute");
            b->gqa_smem = (int)gs;
        }
    }
    ok = ok && !bfail(b, cudaStreamSynchronize(b->st), "batched setup");
    if (!ok) {
        if (err && cap) snprintf(err, cap, "%s", b->msg[0] ? b->msg : "Batched decode setup failed.");
        pkb_destroy(b);
        return NULL;
    }
    return b;
}

extern "C" int pkb_step(PkbCtx *b, const int *tokens, const int *pos, const int *seq_ids, int n, int *next,
                        float *logits)
{
    const int B = bt::BMAX;
    cudaSetDevice(b->device);
    memcpy(b->io_h, tokens, (size_t)n * 4);
    memcpy(b->io_h + B, pos, (size_t)n * 4);
    memcpy(b->io_h + 2 * B, seq_ids, (size_t)n * 4);
    // a tensor-parallel rank assembles the full logits only when asked
    // (every rank of the group must ask alike: the exchanges are collective)
    const int wl = b->world > 1 && logits != NULL ? 1 : 0;
    if (b->exec[wl][n] == NULL) {
        // capture the step for this batch size: input copy, kernels, outputs
        cudaGetLastError();
        if (bfail(b, cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal), "capture")) return 0;
        cudaMemcpyAsync(b->io_d, b->io_h, (size_t)(3 * B) * 4, cudaMemcpyHostToDevice, b->st);
        const int ok = enqueue_step(b, n, wl);
        cudaGraph_t g = NULL;
        const cudaError_t e = cudaStreamEndCapture(b->st, &g);
        if (!ok || bfail(b, e, "capture") ||
            bfail(b, cudaGraphInstantiate(&b->exec[wl][n], g, 0), "graph instantiate")) {
            if (!b->msg[0]) snprintf(b->msg, sizeof(b->msg), "Could not build the batched step.");
            if (g) cudaGraphDestroy(g);
            b->exec[wl][n] = NULL;
            return 0;
        }
        b->graph[wl][n] = g;
    }
    if (bfail(b, cudaGraphLaunch(b->exec[wl][n], b->st), "graph launch") ||
        bfail(b, cudaStreamSynchronize(b->st), "batched step"))
        return 0;
    if (b->io_h[4 * B] != 0) {
        snprintf(b->msg, sizeof(b->msg), "A device wait of the batched step ran out of time (error word %d).",
                 b->io_h[4 * B]);
        return 0;
    }
    memcpy(next, b->io_h + 3 * B, (size_t)n * 4);
    if (logits != NULL &&
        bfail(b, cudaMemcpy(logits, wl ? b->logits_full : b->logits, (size_t)n * b->m.vocab_size * 4,
                            cudaMemcpyDeviceToHost),
              "logits copy"))
        return 0;
    return 1;
}

extern "C" const char *pkb_error(const PkbCtx *b)
{
    return b ? b->msg : "";
}

extern "C" void pkb_destroy(PkbCtx *b)
{
    if (b == NULL) return;
    cudaSetDevice(b->device);
    for (int w = 0; w < 2; w++) {
        for (int i = 0; i <= bt::BMAX; i++) {
            if (b->exec[w][i]) cudaGraphExecDestroy(b->exec[w][i]);
            if (b->graph[w][i]) cudaGraphDestroy(b->graph[w][i]);
        }
    }
    void *dev[] = {b->kv_alias ? nullptr : b->kc, b->kv_alias ? nullptr : b->vc, b->x, b->xn, b->tmp, b->q, b->att,
                   b->k, b->v, b->g, b->u, b->logits, b->part, b->io_d, b->tag0, b->logits_full,
                   b->mm.xs, b->mm.x2s, b->mm.xinv, b->mm.ypart, b->mm.arrived, b->mm.err};
    for (void *p : dev)
        if (p) cudaFree(p);
    if (b->io_h) cudaFreeHost(b->io_h);
    if (b->ev_fork) cudaEventDestroy(b->ev_fork);
    if (b->ev_join) cudaEventDestroy(b->ev_join);
    if (b->side) cudaStreamDestroy(b->side);
    free(b);
}
