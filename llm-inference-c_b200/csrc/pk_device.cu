// pk_device.cu - sm_100a kernels of the GGUF quantized decode path and the
// device half of the engine (run state, decode-step CUDA graph).
//
// Kernels
//   mv_kernel<PRO, EPI>  streaming fused dequant-matvec. Every warp is an
//                        independent pipeline: lane 0 streams tiles of whole
//                        packed rows from HBM into the warp's shared-memory
//                        ring with cp.async.bulk (1-D TMA) completing on
//                        per-stage mbarriers; all 32 lanes then compute the
//                        tile, one 64-column unit per lane with the
//                        activations in registers, and reduce with shuffles.
//                        The prologue stages x (optionally RMSNorm'ed) in
//                        shared memory while the first tiles are in flight;
//                        the epilogue fuses RoPE + KV append (Q/K/V), the
//                        residual add (Wo, ffn_down), SiLU*up (gate/up
//                        pairs) or logits + greedy argmax.
//   attn_kernel          GQA decode attention over the FP32 KV cache, split
//                        over positions, one CTA per (KV head, split); the
//                        last CTA of a KV head merges the splits.
//   embed_kernel         bit-exact decode of one token-embedding row.
//   dequant_kernel       bit-exact row decode (the gguf_weight_dequantize_row
//                        seam) and fp16 table conversion.
//
// Reference counterparts: src/gguf_model.c:441-771 (matvec kernels and
// dispatch), src/gguf_forward.c:159-313 (layer loop), src/sampler.c:39-52
// (greedy).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pk_dev.h"
#include "pk_quant.cuh"
#include "../../include/gguf_cuda.h"

namespace pk {

constexpr int RMAX = 8;          // rows per tile (per matrix)
constexpr int MV_WARPS = 8;      // warps per CTA of mv_kernel
constexpr int XPAD = 68;         // padded floats per 64-column unit in smem
constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;  // ~2 s at 2 GHz

enum { PRO_PLAIN = 0, PRO_NORM = 1 };
enum { EPI_STORE = 0, EPI_ADD = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };
enum { KIND_PLAIN = 0, KIND_Q = 1, KIND_K = 2, KIND_V = 3 };
enum { ERR_TIMEOUT_MV = 1, ERR_TIMEOUT_ATTN = 2 };

// ------------------------------------------------------------------ //
// PTX helpers: mbarrier + 1-D bulk copy                              //
// ------------------------------------------------------------------ //

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar`, giving up after WAIT_LIMIT_CYCLES.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    }
    return true;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// Float -> uint32 whose unsigned order is the float order.
__device__ __forceinline__ uint32_t order_key(float f)
{
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ------------------------------------------------------------------ //
// Streaming matvec                                                   //
// ------------------------------------------------------------------ //

struct MvSeg {
    const uint8_t *w;   // row 0 of the (first) matrix
    const uint8_t *w2;  // row 0 of the paired matrix (EPI_SWIGLU) or null
    uint64_t rb;        // bytes per row
    int rows, type, R, tile0, kind;
};

struct MvArgs {
    MvSeg seg[3];
    int nseg, ntiles;
    int cols, nunits;
    const float *xin;
    const float *norm;
    float eps;
    float *y;
    // Q/K/V epilogue
    float *q, *kc, *vc;
    const float *rope_cs;
    const int *step;
    int hs, rope_dim, kv_dim, seq_len, layer;
    unsigned long long *amax;  // [0] packed argmax, [1] non-finite flag
    int stages, stage_bytes, bar_bytes, xs_bytes;
    int *err;
};

__device__ __forceinline__ const MvSeg &find_seg(const MvArgs &a, int t)
{
    if (a.nseg > 2 && t >= a.seg[2].tile0) return a.seg[2];
    if (a.nseg > 1 && t >= a.seg[1].tile0) return a.seg[1];
    return a.seg[0];
}

// Bytes [st, st + n) of global memory land at buf + (st & 15): the 16-byte
// aligned body goes through the bulk-copy engine, the sub-16-byte tail (only
// a matrix's last row can end unaligned) through plain loads by this lane,
// so nothing past the end of the matrix is read. Returns the bulk bytes.
struct Span {
    uintptr_t a0;
    uint32_t bulk, tail;
};

__device__ __forceinline__ Span make_span(uintptr_t st, uint64_t n)
{
    Span sp;
    sp.a0 = st & ~(uintptr_t)15;
    const uintptr_t a1 = (st + n) & ~(uintptr_t)15;
    sp.bulk = a1 > sp.a0 ? (uint32_t)(a1 - sp.a0) : 0u;
    sp.tail = (uint32_t)(st + n - (sp.a0 + sp.bulk));
    return sp;
}

__device__ __forceinline__ void fill_span(const Span &sp, uint8_t *buf, uint64_t *bar)
{
    if (sp.bulk) bulk_g2s(buf, reinterpret_cast<const void *>(sp.a0), sp.bulk, bar);
    const uint8_t *t = reinterpret_cast<const uint8_t *>(sp.a0 + sp.bulk);
    for (uint32_t i = 0; i < sp.tail; i++) buf[sp.bulk + i] = t[i];
}

// Issue the copies of tile t into `buf` (lane 0); completes on `bar`.
__device__ __forceinline__ void issue_tile(const MvArgs &a, int t, uint8_t *buf, uint64_t *bar)
{
    const MvSeg &s = find_seg(a, t);
    const int r0 = (t - s.tile0) * s.R;
    const int nr = min(s.R, s.rows - r0);
    const uint64_t n = (uint64_t)nr * s.rb;
    const Span sa = make_span(reinterpret_cast<uintptr_t>(s.w) + (uintptr_t)r0 * s.rb, n);
    if (s.w2 != nullptr) {
        const Span sb = make_span(reinterpret_cast<uintptr_t>(s.w2) + (uintptr_t)r0 * s.rb, n);
        mbar_expect_tx(bar, sa.bulk + sb.bulk);
        fill_span(sa, buf, bar);
        fill_span(sb, buf + a.stage_bytes / 2, bar);
    } else {
        mbar_expect_tx(bar, sa.bulk);
        fill_span(sa, buf, bar);
    }
}

__device__ __forceinline__ int xpad(int i)
{
    return (i >> 6) * XPAD + (i & 63);
}

// Accumulate the tile's rows (and paired rows) over this lane's units.
template <int T, bool PAIR>
__device__ __forceinline__ void tile_units(const uint8_t *ra, const uint8_t *rb2, uint64_t rbytes, int nr,
                                           int nunits, int cols, const float *xs, float *acc, float *acc2,
                                           int lane)
{
    const int nblk = cols / block_weights(T);
    for (int u = lane; u < nunits; u += 32) {
        float xr[64];
        const float4 *xp = reinterpret_cast<const float4 *>(xs + u * XPAD);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const float4 v = xp[k];
            xr[4 * k] = v.x;
            xr[4 * k + 1] = v.y;
            xr[4 * k + 2] = v.z;
            xr[4 * k + 3] = v.w;
        }
        float xlo = 0.0f, xhi = 0.0f;
        if (T == T_Q4_K || T == T_Q5_K) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
                xlo += xr[i];
                xhi += xr[32 + i];
            }
        }
#pragma unroll
        for (int i = 0; i < RMAX; i++) {
            if (i < nr) {
                const uint8_t *row = ra + (size_t)i * rbytes;
                float v;
                if (T == T_Q4_K) v = unit_q4k(row, u, xr, xlo, xhi);
                else if (T == T_Q5_K) v = unit_q5k(row, u, xr, xlo, xhi);
                else if (T == T_Q6_K) v = unit_q6k(row, u, xr);
                else if (T == T_Q4_0) v = unit_q4_0(row, u, nblk, xr);
                else if (T == T_Q8_0) v = unit_q8_0(row, u, nblk, xr);
                else v = unit_float(T, row, u, cols, xr);
                acc[i] += v;
                if (PAIR) {
                    const uint8_t *row2 = rb2 + (size_t)i * rbytes;
                    float v2;
                    if (T == T_Q4_K) v2 = unit_q4k(row2, u, xr, xlo, xhi);
                    else if (T == T_Q5_K) v2 = unit_q5k(row2, u, xr, xlo, xhi);
                    else if (T == T_Q6_K) v2 = unit_q6k(row2, u, xr);
                    else if (T == T_Q4_0) v2 = unit_q4_0(row2, u, nblk, xr);
                    else if (T == T_Q8_0) v2 = unit_q8_0(row2, u, nblk, xr);
                    else v2 = unit_float(T, row2, u, cols, xr);
                    acc2[i] += v2;
                }
            }
        }
    }
}

template <bool PAIR>
__device__ __forceinline__ void tile_dispatch(int type, const uint8_t *ra, const uint8_t *rb2, uint64_t rbytes,
                                              int nr, int nunits, int cols, const float *xs, float *acc,
                                              float *acc2, int lane)
{
    switch (type) {
    case T_Q4_K: tile_units<T_Q4_K, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    case T_Q5_K: tile_units<T_Q5_K, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    case T_Q6_K: tile_units<T_Q6_K, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    case T_Q4_0: tile_units<T_Q4_0, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    case T_Q8_0: tile_units<T_Q8_0, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    case T_F32: tile_units<T_F32, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    case T_F16: tile_units<T_F16, PAIR>(ra, rb2, rbytes, nr, nunits, cols, xs, acc, acc2, lane); break;
    default: break;
    }
}

// Stage the input vector in shared memory (padded per 64-column unit),
// RMSNorm'ed as src/gguf_forward.c:24-40 when PRO == PRO_NORM.
template <int PRO>
__device__ __forceinline__ void stage_x(const MvArgs &a, float *xs)
{
    __shared__ float red[32];
    __shared__ float scale_sh;
    const int n = a.cols, tid = threadIdx.x, nt = blockDim.x;
    float sc = 1.0f;
    if (PRO == PRO_NORM) {
        float ss = 0.0f;
        for (int i = tid; i < n; i += nt) {
            const float v = a.xin[i];
            ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid < 32) {
            float v = tid < (nt >> 5) ? red[tid] : 0.0f;
            v = warp_sum(v);
            if (tid == 0) {
                float m = __fdiv_rn(v, (float)n);
                m = __fadd_rn(m, a.eps);
                scale_sh = __fdiv_rn(1.0f, __fsqrt_rn(m));
            }
        }
        __syncthreads();
        sc = scale_sh;
    }
    for (int i = tid; i < a.nunits * 64; i += nt) {
        float v = 0.0f;
        if (i < n) {
            v = a.xin[i];
            if (PRO == PRO_NORM) v = __fmul_rn(a.norm[i], __fmul_rn(sc, v));
        }
        xs[xpad(i)] = v;
    }
    __syncthreads();
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(MV_WARPS * 32, 1) mv_kernel(const __grid_constant__ MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool PAIR = (EPI == EPI_SWIGLU);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = blockDim.x >> 5;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * a.stages;
    float *xs = reinterpret_cast<float *>(smem + a.bar_bytes);
    uint8_t *ring = smem + a.bar_bytes + a.xs_bytes + (size_t)warp * a.stages * a.stage_bytes;

    if (lane == 0) {
        for (int s = 0; s < a.stages; s++) mbar_init(bars + s, 1);
        fence_mbar_init();
    }
    __syncwarp();

    const int gw = blockIdx.x * W + warp, NW = gridDim.x * W;
    const int mine = a.ntiles > gw ? (a.ntiles - 1 - gw) / NW + 1 : 0;
    int issued = 0;
    // Weights do not depend on x: start streaming before staging x.
    if (lane == 0) {
        for (; issued < mine && issued < a.stages - 1; issued++) {
            issue_tile(a, gw + issued * NW, ring + (issued % a.stages) * a.stage_bytes, bars + issued % a.stages);
        }
    }
    stage_x<PRO>(a, xs);

    for (int k = 0; k < mine; k++) {
        if (lane == 0 && issued < mine) {
            issue_tile(a, gw + issued * NW, ring + (issued % a.stages) * a.stage_bytes, bars + issued % a.stages);
            issued++;
        }
        const int stg = k % a.stages;
        if (!mbar_wait_bounded(bars + stg, (uint32_t)((k / a.stages) & 1))) {
            if (lane == 0) atomicOr(a.err, ERR_TIMEOUT_MV);
            return;
        }
        const int t = gw + k * NW;
        const MvSeg &s = find_seg(a, t);
        const int r0 = (t - s.tile0) * s.R;
        const int nr = min(s.R, s.rows - r0);
        const uint8_t *buf = ring + stg * a.stage_bytes;
        const uint8_t *ra = buf + ((reinterpret_cast<uintptr_t>(s.w) + (uintptr_t)r0 * s.rb) & 15);
        const uint8_t *rb2 =
            PAIR ? buf + a.stage_bytes / 2 + ((reinterpret_cast<uintptr_t>(s.w2) + (uintptr_t)r0 * s.rb) & 15)
                 : nullptr;
        float acc[RMAX], acc2[RMAX];
#pragma unroll
        for (int i = 0; i < RMAX; i++) {
            acc[i] = 0.0f;
            acc2[i] = 0.0f;
        }
        tile_dispatch<PAIR>(s.type, ra, rb2, s.rb, nr, a.nunits, a.cols, xs, acc, acc2, lane);
#pragma unroll
        for (int i = 0; i < RMAX; i++) {
            acc[i] = warp_sum(acc[i]);
            if (PAIR) acc2[i] = warp_sum(acc2[i]);
        }
        if (lane == 0) {
            if (EPI == EPI_QKV) {
                const int pos = a.step[1];
                const size_t cache_row = ((size_t)a.layer * a.seq_len + pos) * a.kv_dim;
#pragma unroll
                for (int i = 0; i < RMAX; i += 2) {
                    if (i < nr) {
                        const int r = r0 + i;
                        float v0 = acc[i], v1 = acc[i + 1];
                        const int d = r % a.hs;
                        if (s.kind != KIND_V && d < a.rope_dim) {
                            // rope_head, src/gguf_forward.c:50-66 (cos/sin from the host table)
                            const float c = a.rope_cs[(size_t)pos * a.rope_dim + d];
                            const float sn = a.rope_cs[(size_t)pos * a.rope_dim + d + 1];
                            const float n0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, sn));
                            const float n1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, c));
                            v0 = n0;
                            v1 = n1;
                        }
                        float *dst = s.kind == KIND_Q ? a.q + r : (s.kind == KIND_K ? a.kc : a.vc) + cache_row + r;
                        dst[0] = v0;
                        dst[1] = v1;
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < RMAX; i++) {
                    if (i < nr) {
                        const int r = r0 + i;
                        if (EPI == EPI_STORE) {
                            a.y[r] = acc[i];
                        } else if (EPI == EPI_ADD) {
                            a.y[r] = __fadd_rn(a.y[r], acc[i]);
                        } else if (EPI == EPI_SWIGLU) {
                            const float g = acc[i];
                            a.y[r] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), acc2[i]);
                        } else if (EPI == EPI_LOGITS) {
                            const float v = acc[i];
                            a.y[r] = v;
                            if (isfinite(v)) {
                                atomicMax(a.amax, ((unsigned long long)order_key(v) << 32) |
                                                      (unsigned long long)(0xFFFFFFFFu - (uint32_t)r));
                            } else {
                                atomicOr(a.amax + 1, 1ull);
                            }
                        }
                    }
                }
            }
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------ //
// Launch configuration                                               //
// ------------------------------------------------------------------ //

struct MvPlan {
    MvArgs a;
    dim3 grid, block;
    size_t smem;
    void (*fn)(MvArgs);
};

template <int PRO, int EPI>
static void *mv_fn()
{
    return reinterpret_cast<void *>(&mv_kernel<PRO, EPI>);
}

static int g_sm_count = 0;

// Choose rows per tile, ring depth and grid for one launch. segs[i].w/w2,
// rb, rows, type, kind must be filled. Returns 0 if it cannot fit.
static int plan_mv(MvArgs &a, int nseg, bool pair, bool even_rows, void *fn, dim3 &grid, size_t &smem)
{
    const int mult = pair ? 2 : 1;
    const int target = 4096;
    int stage = 0, t = 0;
    for (int i = 0; i < nseg; i++) {
        MvSeg &s = a.seg[i];
        int R = (int)(target / (s.rb * mult));
        if (R < 1) R = 1;
        if (R > RMAX) R = RMAX;
        if (even_rows) {
            R &= ~1;
            if (R < 2) R = 2;
        }
        s.R = R;
        s.tile0 = t;
        t += (s.rows + R - 1) / R;
        int sb = (int)(((uint64_t)R * s.rb + 32 + 127) / 128 * 128) * mult;
        if (sb > stage) stage = sb;
    }
    a.nseg = nseg;
    a.ntiles = t;
    a.stage_bytes = stage;
    a.nunits = (a.cols + 63) / 64;
    a.xs_bytes = (a.nunits * XPAD * 4 + 127) / 128 * 128;
    for (int stages = 3; stages >= 2; stages--) {
        a.stages = stages;
        a.bar_bytes = (MV_WARPS * stages * 8 + 127) / 128 * 128;
        smem = (size_t)a.bar_bytes + a.xs_bytes + (size_t)MV_WARPS * stages * stage;
        if (smem <= 220 * 1024) break;
    }
    if (smem > 220 * 1024) return 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, MV_WARPS * 32, smem) != cudaSuccess ||
        per_sm < 1)
        return 0;
    if (g_sm_count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    }
    const int want = (a.ntiles + MV_WARPS - 1) / MV_WARPS;
    int g = g_sm_count * per_sm;
    if (want < g) g = want;
    if (g < 1) g = 1;
    grid = dim3(g);
    return 1;
}

// ------------------------------------------------------------------ //
// Attention                                                          //
// ------------------------------------------------------------------ //

struct AttnArgs {
    const float *q, *kc, *vc;
    float *out, *part;
    unsigned *count;
    const int *step;
    int layer, seq_len, kv_dim, hs, kv_mul, nsplit, chunk_max;
    float scale;
};

// Grid (n_kv_heads, nsplit). CTA (g, s) scores positions of split s for
// the kv_mul query heads sharing KV head g (reads each K/V row once),
// src/gguf_forward.c:228-267 with softmax of src/transformer.c:85-109 done
// as a split max/sum merge.
__global__ void __launch_bounds__(256) attn_kernel(const __grid_constant__ AttnArgs a)
{
    extern __shared__ __align__(16) float sm[];
    const int g = blockIdx.x, s = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int hs = a.hs, km = a.kv_mul;
    float *qs = sm;                      // km * hs
    float *sc = sm + km * hs;            // km * chunk_max
    __shared__ int last_sh;

    const int n = a.step[1] + 1;
    const int chunk = (n + a.nsplit - 1) / a.nsplit;
    const int t0 = s * chunk, t1 = min(n, t0 + chunk);
    const int cnt = t1 > t0 ? t1 - t0 : 0;

    for (int i = tid; i < km * hs; i += blockDim.x) qs[i] = a.q[(size_t)g * km * hs + i];
    __syncthreads();

    const size_t lbase = (size_t)a.layer * a.seq_len * a.kv_dim + (size_t)g * hs;
    const float *K = a.kc + lbase;
    const float *V = a.vc + lbase;
    for (int t = warp; t < cnt; t += nw) {
        const float *kr = K + (size_t)(t0 + t) * a.kv_dim;
        for (int hh = 0; hh < km; hh++) {
            float p = 0.0f;
            for (int d = lane; d < hs; d += 32) p = fmaf(qs[hh * hs + d], kr[d], p);
            p = warp_sum(p);
            if (lane == 0) sc[hh * a.chunk_max + t] = p * a.scale;
        }
    }
    __syncthreads();
    // Per head: max, exponentials, sum. One warp per head.
    float *pm = sc + km * a.chunk_max;  // km maxima
    float *pl = pm + km;                // km sums
    for (int hh = warp; hh < km; hh += nw) {
        float m = -INFINITY;
        for (int t = lane; t < cnt; t += 32) m = fmaxf(m, sc[hh * a.chunk_max + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < cnt; t += 32) {
            const float e = expf(sc[hh * a.chunk_max + t] - m);
            sc[hh * a.chunk_max + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            pm[hh] = m;
            pl[hh] = l;
        }
    }
    __syncthreads();
    // Unnormalised partial outputs.
    const int stride = hs + 2;
    for (int i = tid; i < km * hs; i += blockDim.x) {
        const int hh = i / hs, d = i % hs;
        float o = 0.0f;
        for (int t = 0; t < cnt; t++) o = fmaf(sc[hh * a.chunk_max + t], V[(size_t)(t0 + t) * a.kv_dim + d], o);
        float *P = a.part + ((size_t)(g * km + hh) * a.nsplit + s) * stride;
        P[2 + d] = o;
        if (d == 0) {
            P[0] = cnt ? pm[hh] : -INFINITY;
            P[1] = cnt ? pl[hh] : 0.0f;
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_sh = (atomicAdd(a.count + g, 1u) == (unsigned)(a.nsplit - 1));
    __syncthreads();
    if (!last_sh) return;
    __threadfence();
    // Merge the splits in split order.
    for (int i = tid; i < km * hs; i += blockDim.x) {
        const int hh = i / hs, d = i % hs;
        const float *P = a.part + (size_t)(g * km + hh) * a.nsplit * stride;
        float M = -INFINITY;
        for (int j = 0; j < a.nsplit; j++) {
            if (__ldcg(P + (size_t)j * stride + 1) > 0.0f) M = fmaxf(M, __ldcg(P + (size_t)j * stride));
        }
        float L = 0.0f, O = 0.0f;
        for (int j = 0; j < a.nsplit; j++) {
            const float l = __ldcg(P + (size_t)j * stride + 1);
            if (l > 0.0f) {
                const float f = expf(__ldcg(P + (size_t)j * stride) - M);
                L = fmaf(l, f, L);
                O = fmaf(__ldcg(P + (size_t)j * stride + 2 + d), f, O);
            }
        }
        a.out[(size_t)(g * km + hh) * hs + d] = O / L;
    }
    if (tid == 0) a.count[g] = 0;
}

// ------------------------------------------------------------------ //
// Embedding row, dequantization                                      //
// ------------------------------------------------------------------ //

// x = row `token` of the embedding table, decoded exactly; also clears the
// argmax slots of this step.
__global__ void embed_kernel(const uint8_t *embd, uint64_t rb, int type, int dim, const int *step, float *x,
                             unsigned long long *amax)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c == 0) {
        amax[0] = 0ull;
        amax[1] = 0ull;
    }
    if (c < dim) x[c] = decode_col(type, embd + (size_t)step[0] * rb, c);
}

// End of a decode step: the greedy token becomes the next step's input
// (token, pos + 1) and is appended to the device token log. A non-finite
// logit or an empty argmax stops the chain with token 0 and a flag.
__global__ void finish_kernel(int *step, const unsigned long long *amax, int *tokens, int cap, int *err)
{
    const unsigned long long k = amax[0];
    int tok = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    if (amax[1] != 0ull || k == 0ull) {
        tok = -1;
        atomicOr(err, 4);
    }
    const int n = step[2];
    if (n < cap) tokens[n] = tok;
    step[0] = tok < 0 ? 0 : tok;
    step[1] = step[1] + 1;
    step[2] = n + 1;
}

__global__ void dequant_kernel(const uint8_t *w, uint64_t rb, int type, uint64_t rows, uint64_t cols,
                               float *out)
{
    const uint64_t n = rows * cols;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / cols, c = i % cols;
        out[i] = decode_col(type, w + r * rb, (int)c);
    }
}

__global__ void fp16_table_kernel(float *out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < 65536) out[i] = h2f((uint32_t)i);
}

}  // namespace pk

using namespace pk;

// ================================================================== //
// Public device-level seam (include/gguf_cuda.h)                     //
// ================================================================== //

static int supported_type(uint32_t t)
{
    return t == T_F32 || t == T_F16 || t == T_Q4_0 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

static int weight_ok(const GGUFWeight *w)
{
    if (w == NULL || w->data == NULL || !supported_type(w->type) || w->rows == 0 || w->cols == 0) return 0;
    const uint64_t bw = (uint64_t)block_weights((int)w->type);
    if (w->cols % bw) return 0;
    if (w->row_bytes != w->cols / bw * (uint64_t)block_bytes((int)w->type)) return 0;
    if (w->rows > 0x7FFFFFFFull || w->cols > 0x7FFFFFFFull) return 0;
    if (((uintptr_t)w->data & 15) != 0) return 0;  // rows are staged by 16-byte bulk copies
    return 1;
}

extern "C" int gguf_cuda_matvec(const GGUFWeight *weight, const float *x, float *out, void *stream)
{
    if (!weight_ok(weight) || x == NULL || out == NULL || (const void *)x == (const void *)out) return 0;
    MvArgs a;
    memset(&a, 0, sizeof(a));
    a.seg[0].w = (const uint8_t *)weight->data;
    a.seg[0].rb = weight->row_bytes;
    a.seg[0].rows = (int)weight->rows;
    a.seg[0].type = (int)weight->type;
    a.cols = (int)weight->cols;
    a.xin = x;
    a.y = out;
    static int *d_err = NULL;
    if (d_err == NULL && cudaMalloc(&d_err, sizeof(int)) != cudaSuccess) return 0;
    a.err = d_err;
    void *fn = mv_fn<PRO_PLAIN, EPI_STORE>();
    dim3 grid;
    size_t smem;
    if (!plan_mv(a, 1, false, false, fn, grid, smem)) return 0;
    mv_kernel<PRO_PLAIN, EPI_STORE><<<grid, MV_WARPS * 32, smem, (cudaStream_t)stream>>>(a);
    return cudaGetLastError() == cudaSuccess;
}

extern "C" int gguf_cuda_dequantize_rows(const GGUFWeight *weight, uint64_t row0, uint64_t nrows, float *out,
                                         void *stream)
{
    if (!weight_ok(weight) || out == NULL || row0 >= weight->rows || nrows > weight->rows - row0) return 0;
    if (nrows == 0) return 1;
    const uint64_t n = nrows * weight->cols;
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    dequant_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint8_t *)weight->data + row0 * weight->row_bytes,
                                                              weight->row_bytes, (int)weight->type, nrows,
                                                              weight->cols, out);
    return cudaGetLastError() == cudaSuccess;
}

extern "C" int gguf_cuda_fp16_table(float *out65536, void *stream)
{
    if (out65536 == NULL) return 0;
    fp16_table_kernel<<<256, 256, 0, (cudaStream_t)stream>>>(out65536);
    return cudaGetLastError() == cudaSuccess;
}

// ================================================================== //
// Device half of the engine                                          //
// ================================================================== //

struct PkdCtx {
    int device;
    cudaStream_t stream;
    uint8_t *arena;
    uint64_t arena_bytes;
    void *staging;  // pinned upload staging
    // run state
    float *x, *xb, *q, *hb, *logits, *kc, *vc, *part, *norms, *rope_cs;
    unsigned *count;
    int *step_d, *err_d, *tokens_d;
    int tokens_cap;
    unsigned long long *amax_d;
    cudaEvent_t ev0, ev1;
    // pinned host mirrors
    int *step_h;
    float *logits_h;
    unsigned long long *amax_h;
    int *err_h;
    int vocab, failed;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    char msg[256];
};

static int cuda_fail(PkdCtx *c, cudaError_t e, const char *what, char *err, size_t cap)
{
    if (e == cudaSuccess) return 0;
    if (c) snprintf(c->msg, sizeof(c->msg), "%s: %s", what, cudaGetErrorString(e));
    if (err && cap) snprintf(err, cap, "CUDA %s failed: %s", what, cudaGetErrorString(e));
    return 1;
}

extern "C" PkdCtx *pkd_create(int device, uint64_t arena_bytes, char *err, size_t cap)
{
    PkdCtx *c = (PkdCtx *)calloc(1, sizeof(PkdCtx));
    if (c == NULL) {
        if (err && cap) snprintf(err, cap, "Out of memory.");
        return NULL;
    }
    c->device = device;
    if (cuda_fail(c, cudaSetDevice(device), "cudaSetDevice", err, cap) ||
        cuda_fail(c, cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate", err, cap) ||
        cuda_fail(c, cudaMalloc((void **)&c->arena, arena_bytes + 256), "cudaMalloc(weights)", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->staging, 64u << 20), "cudaMallocHost(staging)", err, cap)) {
        pkd_destroy(c);
        return NULL;
    }
    c->arena_bytes = arena_bytes;
    cudaMemsetAsync(c->arena, 0, arena_bytes + 256, c->stream);
    return c;
}

extern "C" int pkd_upload(PkdCtx *c, uint64_t offset, const void *src, uint64_t bytes, char *err, size_t cap)
{
    if (c == NULL || offset + bytes > c->arena_bytes) {
        if (err && cap) snprintf(err, cap, "Upload outside the weight arena.");
        return 0;
    }
    const uint64_t chunk = 32u << 20;
    const uint8_t *s = (const uint8_t *)src;
    for (uint64_t done = 0; done < bytes;) {
        const uint64_t n = bytes - done < chunk ? bytes - done : chunk;
        // Two halves of the pinned staging buffer alternate.
        uint8_t *stg = (uint8_t *)c->staging + ((done / chunk) & 1) * chunk;
        if (cuda_fail(c, cudaStreamSynchronize(c->stream), "upload sync", err, cap)) return 0;
        memcpy(stg, s + done, n);
        if (cuda_fail(c, cudaMemcpyAsync(c->arena + offset + done, stg, n, cudaMemcpyHostToDevice, c->stream),
                      "upload copy", err, cap))
            return 0;
        done += n;
    }
    return 1;
}

static void fill_seg(MvSeg &s, const PkdCtx *c, const PkdTensor &t, int kind)
{
    s.w = c->arena + t.offset;
    s.w2 = nullptr;
    s.rb = t.row_bytes;
    s.rows = (int)t.rows;
    s.type = (int)t.type;
    s.kind = kind;
}

template <int PRO, int EPI>
static int launch_mv(MvArgs &a, int nseg, bool even, cudaStream_t st)
{
    void *fn = mv_fn<PRO, EPI>();
    dim3 grid;
    size_t smem;
    if (!plan_mv(a, nseg, EPI == EPI_SWIGLU, even, fn, grid, smem)) return 0;
    mv_kernel<PRO, EPI><<<grid, MV_WARPS * 32, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess;
}

// Record one decode step on c->stream (used under stream capture).
static int record_step(PkdCtx *c, const PkdModel *m)
{
    const int dim = m->dim, hs = m->dim / m->n_heads;
    const int kvd = hs * m->n_kv_heads, km = m->n_heads / m->n_kv_heads;
    cudaStream_t st = c->stream;
    embed_kernel<<<(dim + 255) / 256, 256, 0, st>>>(c->arena + m->embd.offset, m->embd.row_bytes,
                                                    (int)m->embd.type, dim, c->step_d, c->x, c->amax_d);
    if (cudaGetLastError() != cudaSuccess) return 0;

    int nsplit = (2 * (g_sm_count ? g_sm_count : 148) + m->n_kv_heads - 1) / m->n_kv_heads;
    if (nsplit > m->seq_len) nsplit = m->seq_len;
    const int chunk_max = (m->seq_len + nsplit - 1) / nsplit;
    const size_t attn_smem = (size_t)(km * hs + km * chunk_max + 2 * km) * sizeof(float);

    for (int l = 0; l < m->n_layers; l++) {
        MvArgs a;
        memset(&a, 0, sizeof(a));
        a.cols = dim;
        a.xin = c->x;
        a.norm = c->norms + (size_t)(2 * l) * dim;
        a.eps = m->rms_eps;
        a.q = c->q;
        a.kc = c->kc;
        a.vc = c->vc;
        a.rope_cs = c->rope_cs;
        a.step = c->step_d;
        a.hs = hs;
        a.rope_dim = m->rope_dim;
        a.kv_dim = kvd;
        a.seq_len = m->seq_len;
        a.layer = l;
        a.err = c->err_d;
        fill_seg(a.seg[0], c, m->wq[l], KIND_Q);
        fill_seg(a.seg[1], c, m->wk[l], KIND_K);
        fill_seg(a.seg[2], c, m->wv[l], KIND_V);
        if (!launch_mv<PRO_NORM, EPI_QKV>(a, 3, true, st)) return 0;

        AttnArgs at;
        at.q = c->q;
        at.kc = c->kc;
        at.vc = c->vc;
        at.out = c->xb;
        at.part = c->part;
        at.count = c->count;
        at.step = c->step_d;
        at.layer = l;
        at.seq_len = m->seq_len;
        at.kv_dim = kvd;
        at.hs = hs;
        at.kv_mul = km;
        at.nsplit = nsplit;
        at.chunk_max = chunk_max;
        at.scale = m->att_scale;
        attn_kernel<<<dim3(m->n_kv_heads, nsplit), 128, attn_smem, st>>>(at);
        if (cudaGetLastError() != cudaSuccess) return 0;

        MvArgs o;
        memset(&o, 0, sizeof(o));
        o.cols = dim;
        o.xin = c->xb;
        o.y = c->x;
        o.err = c->err_d;
        fill_seg(o.seg[0], c, m->wo[l], KIND_PLAIN);
        if (!launch_mv<PRO_PLAIN, EPI_ADD>(o, 1, false, st)) return 0;

        MvArgs f;
        memset(&f, 0, sizeof(f));
        f.cols = dim;
        f.xin = c->x;
        f.norm = c->norms + (size_t)(2 * l + 1) * dim;
        f.eps = m->rms_eps;
        f.y = c->hb;
        f.err = c->err_d;
        fill_seg(f.seg[0], c, m->gate[l], KIND_PLAIN);
        f.seg[0].w2 = c->arena + m->up[l].offset;
        if (m->gate[l].type != m->up[l].type) return 0;  // caller falls back (not in our models)
        if (!launch_mv<PRO_NORM, EPI_SWIGLU>(f, 1, false, st)) return 0;

        MvArgs dn;
        memset(&dn, 0, sizeof(dn));
        dn.cols = m->hidden_dim;
        dn.xin = c->hb;
        dn.y = c->x;
        dn.err = c->err_d;
        fill_seg(dn.seg[0], c, m->down[l], KIND_PLAIN);
        if (!launch_mv<PRO_PLAIN, EPI_ADD>(dn, 1, false, st)) return 0;
    }
    MvArgs lg;
    memset(&lg, 0, sizeof(lg));
    lg.cols = dim;
    lg.xin = c->x;
    lg.norm = c->norms + (size_t)(2 * m->n_layers) * dim;
    lg.eps = m->rms_eps;
    lg.y = c->logits;
    lg.amax = c->amax_d;
    lg.err = c->err_d;
    fill_seg(lg.seg[0], c, m->output, KIND_PLAIN);
    if (!launch_mv<PRO_NORM, EPI_LOGITS>(lg, 1, false, st)) return 0;
    finish_kernel<<<1, 1, 0, st>>>(c->step_d, c->amax_d, c->tokens_d, c->tokens_cap, c->err_d);
    return cudaGetLastError() == cudaSuccess;
}

extern "C" int pkd_build(PkdCtx *c, const PkdModel *m, char *err, size_t cap)
{
    const size_t dim = (size_t)m->dim, hid = (size_t)m->hidden_dim;
    const size_t hs = dim / (size_t)m->n_heads, kvd = hs * (size_t)m->n_kv_heads;
    const size_t cache = (size_t)m->n_layers * (size_t)m->seq_len * kvd;
    const size_t nnorm = (2 * (size_t)m->n_layers + 1) * dim;
    if (m->gate == NULL || (size_t)m->rope_dim > hs || hs % 2) {
        if (err && cap) snprintf(err, cap, "Unsupported model shape.");
        return 0;
    }
    for (int l = 0; l < m->n_layers; l++) {
        if (m->gate[l].type != m->up[l].type) {
            if (err && cap) snprintf(err, cap, "ffn_gate and ffn_up must share a type.");
            return 0;
        }
    }
    cudaSetDevice(c->device);
    if (g_sm_count == 0) cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, c->device);
    int nsplit = (2 * g_sm_count + m->n_kv_heads - 1) / m->n_kv_heads;
    if (nsplit > m->seq_len) nsplit = m->seq_len;
    const size_t part = (size_t)m->n_heads * nsplit * (hs + 2);
    if (cuda_fail(c, cudaMalloc(&c->x, dim * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->xb, dim * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->q, dim * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->hb, hid * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->logits, (size_t)m->vocab_size * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->kc, cache * 4), "cudaMalloc(KV cache)", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->vc, cache * 4), "cudaMalloc(KV cache)", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->part, part * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->norms, nnorm * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->rope_cs, (size_t)m->seq_len * m->rope_dim * 4 + 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->count, (size_t)m->n_kv_heads * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->step_d, 16), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->err_d, 16), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->amax_d, 16), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->tokens_d, (size_t)m->seq_len * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaEventCreate(&c->ev0), "cudaEventCreate", err, cap) ||
        cuda_fail(c, cudaEventCreate(&c->ev1), "cudaEventCreate", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->step_h, 16), "cudaMallocHost", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->logits_h, (size_t)m->vocab_size * 4), "cudaMallocHost", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->amax_h, 16), "cudaMallocHost", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->err_h, 16), "cudaMallocHost", err, cap)) {
        return 0;
    }
    c->vocab = m->vocab_size;
    c->tokens_cap = m->seq_len;
    cudaStream_t st = c->stream;
    cudaMemsetAsync(c->kc, 0, cache * 4, st);
    cudaMemsetAsync(c->vc, 0, cache * 4, st);
    cudaMemsetAsync(c->count, 0, (size_t)m->n_kv_heads * 4, st);
    cudaMemsetAsync(c->err_d, 0, 16, st);
    cudaMemsetAsync(c->step_d, 0, 16, st);
    // Norm weights decoded once on the device (src/gguf_forward.c:116-144).
    for (int l = 0; l <= m->n_layers; l++) {
        for (int k = 0; k < 2; k++) {
            if (l == m->n_layers && k == 1) break;
            const PkdTensor &t = l == m->n_layers ? m->output_norm : (k == 0 ? m->attn_norm[l] : m->ffn_norm[l]);
            dequant_kernel<<<(m->dim + 255) / 256, 256, 0, st>>>(c->arena + t.offset, t.row_bytes, (int)t.type, 1,
                                                                   (uint64_t)m->dim,
                                                                   c->norms + (size_t)(2 * l + k) * dim);
        }
    }
    if (cuda_fail(c, cudaGetLastError(), "norm decode", err, cap) ||
        cuda_fail(c,
                  cudaMemcpyAsync(c->rope_cs, m->rope_cs, (size_t)m->seq_len * m->rope_dim * 4,
                                  cudaMemcpyHostToDevice, st),
                  "rope upload", err, cap) ||
        cuda_fail(c, cudaStreamSynchronize(st), "build sync", err, cap)) {
        return 0;
    }
    // Capture one decode step as a graph; replays read token/pos from step_d.
    if (cuda_fail(c, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "capture", err, cap)) return 0;
    const int ok = record_step(c, m);
    cudaError_t e = cudaStreamEndCapture(st, &c->graph);
    if (!ok || e != cudaSuccess) {
        if (err && cap) snprintf(err, cap, "Cannot record the decode step (%s).", cudaGetErrorString(e));
        return 0;
    }
    if (cuda_fail(c, cudaGraphInstantiate(&c->exec, c->graph, 0), "graph instantiate", err, cap)) return 0;
    return 1;
}

static int run_step(PkdCtx *c, int token, int pos, int want_logits)
{
    if (c == NULL || c->failed) return 0;
    c->step_h[0] = token;
    c->step_h[1] = pos;
    c->step_h[2] = 0;
    cudaStream_t st = c->stream;
    cudaMemcpyAsync(c->step_d, c->step_h, 12, cudaMemcpyHostToDevice, st);
    cudaGraphLaunch(c->exec, st);
    if (want_logits) cudaMemcpyAsync(c->logits_h, c->logits, (size_t)c->vocab * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(c->amax_h, c->amax_d, 16, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(c->err_h, c->err_d, 4, cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        snprintf(c->msg, sizeof(c->msg), "decode step: %s", cudaGetErrorString(e));
        c->failed = 1;
        return 0;
    }
    if (c->err_h[0] & 4) cudaMemsetAsync(c->err_d, 0, 4, st);  // non-finite logits: a value, not a failure
    if (c->err_h[0] & 3) {
        snprintf(c->msg, sizeof(c->msg), "decode step: device wait timed out (code %d)", c->err_h[0]);
        c->failed = 1;
        return 0;
    }
    return 1;
}

extern "C" float *pkd_forward(PkdCtx *c, int token, int pos)
{
    return run_step(c, token, pos, 1) ? c->logits_h : NULL;
}

extern "C" int pkd_forward_greedy(PkdCtx *c, int token, int pos)
{
    if (!run_step(c, token, pos, 0)) return -2;
    if (c->amax_h[1] != 0ull || c->amax_h[0] == 0ull) return -1;
    return (int)(0xFFFFFFFFu - (uint32_t)(c->amax_h[0] & 0xFFFFFFFFull));
}

extern "C" int pkd_generate_greedy(PkdCtx *c, int token, int pos, int n, int *out, float *device_ms)
{
    if (c == NULL || c->failed || n < 0 || n > c->tokens_cap) return 0;
    c->step_h[0] = token;
    c->step_h[1] = pos;
    c->step_h[2] = 0;
    cudaStream_t st = c->stream;
    cudaMemcpyAsync(c->step_d, c->step_h, 12, cudaMemcpyHostToDevice, st);
    cudaEventRecord(c->ev0, st);
    for (int i = 0; i < n; i++) cudaGraphLaunch(c->exec, st);
    cudaEventRecord(c->ev1, st);
    if (n > 0) cudaMemcpyAsync(out, c->tokens_d, (size_t)n * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(c->err_h, c->err_d, 4, cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        snprintf(c->msg, sizeof(c->msg), "generate: %s", cudaGetErrorString(e));
        c->failed = 1;
        return 0;
    }
    if (c->err_h[0] & 3) {
        snprintf(c->msg, sizeof(c->msg), "generate: device wait timed out (code %d)", c->err_h[0]);
        c->failed = 1;
        return 0;
    }
    if (c->err_h[0] & 4) cudaMemsetAsync(c->err_d, 0, 4, st);  // non-finite logits: reported per token as -1
    if (device_ms != NULL) cudaEventElapsedTime(device_ms, c->ev0, c->ev1);
    return 1;
}

extern "C" const char *pkd_error(const PkdCtx *c)
{
    return c ? c->msg : "";
}

extern "C" void pkd_destroy(PkdCtx *c)
{
    if (c == NULL) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->exec) cudaGraphExecDestroy(c->exec);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    if (c->graph) cudaGraphDestroy(c->graph);
    void *dev[] = {c->arena, c->x, c->xb, c->q, c->hb, c->logits, c->kc, c->vc, c->part,
                   c->norms, c->rope_cs, c->count, c->step_d, c->err_d, c->amax_d, c->tokens_d};
    for (size_t i = 0; i < sizeof(dev) / sizeof(dev[0]); i++) {
        if (dev[i]) cudaFree(dev[i]);
    }
    void *host[] = {c->staging, c->step_h, c->logits_h, c->amax_h, c->err_h};
    for (size_t i = 0; i < sizeof(host) / sizeof(host[0]); i++) {
        if (host[i]) cudaFreeHost(host[i]);
    }
    if (c->stream) cudaStreamDestroy(c->stream);
    free(c);
}
