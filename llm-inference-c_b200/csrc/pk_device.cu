// pk_device.cu - sm_100a kernels of the GGUF quantized decode path and the
// device half of the engine (run state, the decode step).
//
// phase_kernel runs phases of pk_stream.cuh:
//   * persistent (cooperative launch, one CTA per SM): every phase of one
//     decode step - per layer QKV(+RoPE, KV append) | attention | Wo(+residual)
//     | gate/up(+SiLU*up) | down(+residual), then the logits - handing
//     activations over as tagged words (no grid barrier), while each warp's
//     bulk-copy ring streams the following phases' weights. One launch per
//     token.
//   * one phase per launch: the standalone gguf_cuda_matvec, and the step as
//     a sequence of launches (POCKET_CUDA_PERSISTENT=0).
// Small kernels: bit-exact row decode, the fp16 table, the greedy hand-off
// between steps, and a plain fallback matvec for very long F32/F16 rows.
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

#include "../../include/gguf_cuda.h"
#include "pk_dev.h"
#include "pk_quant.cuh"
#include "pk_stream.cuh"

namespace pk {

constexpr int DK_WARPS = 12;      // warps per CTA of phase_kernel
constexpr int RMAX = 8;           // rows per tile (per matrix)
constexpr int SMEM_LIMIT = 227 * 1024;  // shared memory per block (opt-in maximum) of sm_100

int smem_dynamic_max();

struct DecodeArgs {
    Phase one;             // the phase to run when `phases` is null
    const Phase *phases;   // device array of nphases phases (one launch per step)
    int nphases;
    const CopyEnt *copies;  // with `phases`: every warp's weight copies in consumption
    const int *copy_off;    //   order, warp gw's at copies[copy_off[gw] .. copy_off[gw + 1])
    int stages, stage_bytes, bar_bytes, xq_bytes, xs_bytes, attn_bytes;
    const int *step;       // {token, pos, generated count, last token, tag}
    const float *rope_cs;  // RoPE cos/sin table [position][rope_dim]
    int rope_dim;
    int *err;
    // Seam launches (gguf_cuda_matvec and the no-allocation variant): err
    // is the call's abort word (any wait that gives up records itself there
    // and the other waits then stop); the last CTA to finish moves it into
    // err[1], which accumulates until the caller reads it, and clears it, so
    // the next call starts clean. err[2] counts finished CTAs.
    int seam;
    unsigned long long *trace;  // optional: CTA 0's %globaltimer at start, then per phase: after
                                //   staging x, after its work, and again at its end; then
                                //   for every CTA and phase: after staging x, after its work
};

// End of a seam launch: the last CTA moves the abort word into the
// caller-visible accumulated word and clears it (see DecodeArgs::seam).
__device__ __forceinline__ void seam_finish(int *err)
{
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence();  // this CTA's error records precede its count
    if (atomicAdd(err + 2, 1) == (int)gridDim.x - 1) {
        __threadfence();
        const int e = atomicExch(err, 0);
        if (e != 0) atomicOr(err + 1, e);
        atomicExch(err + 2, 0);
    }
}

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// The decode step (or one phase of it). The phases run in order in every
// CTA, with no grid-wide barrier: inputs are tagged words that each CTA
// polls, so a CTA enters a phase when the words it needs carry this step's
// tag, and skips a phase in which it has no tile or item. All CTAs must be
// resident together (cooperative launch), since consumers wait on producers
// in other CTAs; every wait is bounded.
template <unsigned MASK>
__global__ void __launch_bounds__(DK_WARPS * 32, 1) phase_kernel(const __grid_constant__ DecodeArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const Phase *ph = a.phases != nullptr ? a.phases : &a.one;
    const int nph = a.phases != nullptr ? a.nphases : 1;
    const int W = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * W + warp, NW = gridDim.x * W;
    const uint32_t tag = a.step != nullptr ? (uint32_t)a.step[4] : 0u;
    const int token = a.step != nullptr ? a.step[0] : 0, pos = a.step != nullptr ? a.step[1] : 0;
    const bool tracing = a.trace != nullptr && blockIdx.x == 0;
    unsigned long long *ctr =
        a.trace != nullptr ? a.trace + 3 * nph + 1 + (size_t)blockIdx.x * 2 * nph : nullptr;

    Ring r;
    r.bars = reinterpret_cast<uint64_t *>(smem) + warp * a.stages;
    r.buf = smem + a.bar_bytes + a.xs_bytes + (size_t)warp * a.stages * a.stage_bytes;
    r.stages = a.stages;
    r.stage_bytes = a.stage_bytes;
    r.issued = r.consumed = 0;
    r.cp = r.ck = 0;
    r.list = nullptr;
    r.nlist = r.next = 0;
    if (a.phases != nullptr && a.copies != nullptr) {
        const int c0 = a.copy_off[gw];
        r.list = a.copies + c0;
        r.nlist = (uint32_t)(a.copy_off[gw + 1] - c0);
        if (lane == 0 && r.nlist > 0) r.pre = ld_copy(r.list);
    }
    // x digits (matvec phases) and attention scratch share one region
    uint8_t *xq = smem + a.bar_bytes;
    float *xg = reinterpret_cast<float *>(smem + a.bar_bytes + a.xq_bytes);
    float *att = reinterpret_cast<float *>(smem + a.bar_bytes);
    __shared__ unsigned long long cta_amax[2];
    __shared__ float rope[256];  // this position's RoPE cos/sin pairs
    // The decode step's phase descriptors pass through shared memory: the
    // next one is bulk-copied while the current one runs, so no field read
    // during a phase waits on L2.
    __shared__ Phase sph[2];
    __shared__ uint64_t dbar;
    const bool staged_desc = a.phases != nullptr;

    if (lane == 0) {
        for (int s = 0; s < a.stages; s++) mbar_init(r.bars + s, 1);
        if (staged_desc && threadIdx.x == 0) mbar_init(&dbar, 1);
        fence_mbar_init();
    }
    if (staged_desc) {
        __syncthreads();  // dbar is initialised before any thread waits on it
        if (threadIdx.x == 0) {
            mbar_expect_tx(&dbar, (uint32_t)sizeof(Phase));
            bulk_g2s(&sph[0], ph, (uint32_t)sizeof(Phase), &dbar);
        }
    }
    __syncwarp();
    // Weights do not depend on activations: start streaming at once.
    if (lane == 0) {
        if (r.list != nullptr) {
            ring_fill_list(r);
        } else {
            ring_fill(r, ph, nph, gw, W, NW);
        }
    }
    if (tracing && threadIdx.x == 0) a.trace[0] = global_ns();
    if (a.rope_cs != nullptr) {
        const float *row = a.rope_cs + (size_t)pos * a.rope_dim;
        for (int i = threadIdx.x; i < a.rope_dim; i += blockDim.x) rope[i] = row[i];
    }

    for (int pi = 0; pi < nph; pi++) {
        if (staged_desc) {
            // descriptor pi has landed (bounded wait, CTA-uniform outcome)
            const int ok = __syncthreads_and(mbar_wait_bounded(&dbar, (uint32_t)(pi & 1)) ? 1 : 0);
            if (!ok) {
                if (threadIdx.x == 0) atomicOr(a.err, ERR_TIMEOUT_MV);
                break;
            }
            // every thread is done with descriptor pi - 1, whose buffer takes pi + 1
            if (threadIdx.x == 0 && pi + 1 < nph) {
                mbar_expect_tx(&dbar, (uint32_t)sizeof(Phase));
                bulk_g2s(&sph[(pi + 1) & 1], ph + pi + 1, (uint32_t)sizeof(Phase), &dbar);
            }
        }
        const Phase &p = staged_desc ? sph[pi & 1] : ph[pi];
        if (p.kind == PH_MV) {
            if (cta_has_tiles(p, blockIdx.x, W, NW)) {
                // every warp is done with the previous phase's x (the barrier
                // above, when the descriptors are staged)
                if (!staged_desc) __syncthreads();
                if (p.epi == EPI_LOGITS && threadIdx.x == 0) cta_amax[0] = cta_amax[1] = 0ull;
                const float nscale = stage_x(p, a.step, xq, xg, tag, a.err);  // ends with __syncthreads
                if (ctr != nullptr && threadIdx.x == 0) {
                    ctr[2 * pi] = global_ns();
                    if (tracing) a.trace[3 * pi + 1] = ctr[2 * pi];
                }
                float racc = 0.0f;  // a chunked row's running sum
                for (int k = 0;; k++) {
                    const int t = tile_at(p, gw, W, NW, k / p.nchunk);
                    if (t >= p.ntiles) break;
                    const uint32_t slot = r.consumed % (uint32_t)a.stages;
                    const uint32_t par = (r.consumed / (uint32_t)a.stages) & 1u;
                    // warp-uniform: run_tile's shuffles name every lane
                    const bool ok =
                        __all_sync(0xFFFFFFFFu, mbar_wait_or_abort(r.bars + slot, par, a.err));
                    if (!ok) {
                        if (lane == 0) atomicOr(a.err, ERR_TIMEOUT_MV);
                    } else {
                        run_tile<MASK>(p, t, k % p.nchunk, r.buf + slot * a.stage_bytes, xq, xg, token, pos, rope,
                                       tag, a.err, lane, cta_amax, racc, nscale);
                    }
                    __syncwarp();
                    r.consumed++;
                    if (lane == 0 && ok) {
                        if (r.list != nullptr) {
                            ring_fill_list(r);
                        } else {
                            ring_fill(r, ph, nph, gw, W, NW);
                        }
                    }
                }
                if (p.epi == EPI_LOGITS) {
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        if (cta_amax[0] != 0ull) atomicMax(p.amax, cta_amax[0]);
                        if (cta_amax[1] != 0ull) atomicOr(p.amax + 1, 1ull);
                        if (p.world > 1) {
                            // this CTA's logits stores to the other ranks precede its count;
                            // the last CTA publishes the rank's argmax to every rank
                            __threadfence_system();
                            if (atomicAdd(p.done, 1u) == (unsigned)(p.ncta - 1)) {
                                __threadfence();
                                const unsigned long long k = *reinterpret_cast<volatile unsigned long long *>(p.amax);
                                const unsigned long long nf = *reinterpret_cast<volatile unsigned long long *>(p.amax + 1);
                                const uint64_t tg = (uint64_t)tag << 32;
                                for (int q = 0; q < p.world; q++) {
                                    uint64_t *slot = p.keys[q] + (size_t)p.rank * 4;
                                    st_u64_sys(slot, tg | (k >> 32));
                                    st_u64_sys(slot + 1, tg | (k & 0xFFFFFFFFull));
                                    st_u64_sys(slot + 2, tg | (nf != 0ull ? 1ull : 0ull));
                                }
                                *p.done = 0u;
                            }
                        }
                    }
                }
            } else if (ctr != nullptr && threadIdx.x == 0) {
                ctr[2 * pi] = global_ns();
                if (tracing) a.trace[3 * pi + 1] = ctr[2 * pi];
            }
        } else if (p.kind == PH_AR) {
            const int items = (p.own[p.rank] + (int)blockDim.x - 1) / (int)blockDim.x;
            if (ctr != nullptr && threadIdx.x == 0) {
                ctr[2 * pi] = global_ns();
                if (tracing) a.trace[3 * pi + 1] = ctr[2 * pi];
            }
            for (int it = (blockIdx.x + gridDim.x - p.off % gridDim.x) % gridDim.x; it < items; it += gridDim.x) {
                ar_item(p, it, a.step, tag, a.err);
            }
        } else {
            const int n = pos + 1, nh = p.n_kv * p.kv_mul;
            const int span = attn_span(n, p.nsplit_max);
            const int nsplit = (n + span - 1) / span;
            if (ctr != nullptr && threadIdx.x == 0) {
                ctr[2 * pi] = global_ns();
                if (tracing) a.trace[3 * pi + 1] = ctr[2 * pi];
            }
            for (int it = (blockIdx.x + gridDim.x - p.off % gridDim.x) % gridDim.x; it < nh * nsplit;
                 it += gridDim.x) {
                __syncthreads();  // the scratch aliases the previous phase's x
                attn_item(p, it % nh, it / nh, nsplit, n, span, att, tag, a.err);
            }
        }
        if (ctr != nullptr) {
            __syncthreads();
            if (threadIdx.x == 0) {
                ctr[2 * pi + 1] = global_ns();
                if (tracing) a.trace[3 * pi + 2] = a.trace[3 * pi + 3] = ctr[2 * pi + 1];
            }
        }
    }
    if (lane == 0 && r.issued != r.consumed) ring_drain(r);
    if (a.seam) seam_finish(a.err);
}

// End of a decode step: the greedy token becomes the next step's input
// (token, pos + 1) and is appended to the device token log; the argmax
// slots are cleared for the next step. A non-finite logit or an empty
// argmax logs -1 and continues from token 0.
__global__ void finish_kernel(int *step, unsigned long long *amax, int *tokens, int cap, int *err)
{
    const unsigned long long k = amax[0];
    int tok = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    if (amax[1] != 0ull || k == 0ull) {
        tok = -1;
        atomicOr(err, ERR_NONFINITE);
    }
    const int n = step[2];
    if (n < cap) tokens[n] = tok;
    step[3] = tok;  // this step's token (read back by single-step callers)
    step[0] = tok < 0 ? 0 : tok;
    step[1] = step[1] + 1;
    step[2] = n + 1;
    step[4] = step[4] + 1;  // the next step's tag
    amax[0] = 0ull;
    amax[1] = 0ull;
}

typedef void (*PhaseFn)(DecodeArgs);

// The compiled phase_kernel variants: one per format for the device seam,
// and format sets of common GGUF mixes for the decode step (Q4_K_M:
// Q4_K + Q6_K; K-quant mixes with Q5_K and Q8_0; legacy Q4_0/Q8_0; float),
// then everything.
struct Variant {
    unsigned mask;
    PhaseFn fn;
};
#define PK_VARIANT(M) {(M), phase_kernel<(M)>}
static const Variant VARIANTS[] = {
    PK_VARIANT(tbit(T_Q4_K)),
    PK_VARIANT(tbit(T_Q5_K)),
    PK_VARIANT(tbit(T_Q6_K)),
    PK_VARIANT(tbit(T_Q4_0)),
    PK_VARIANT(tbit(T_Q8_0)),
    PK_VARIANT(tbit(T_F32)),
    PK_VARIANT(tbit(T_F16)),
    PK_VARIANT(tbit(T_Q4_K) | tbit(T_Q6_K)),
    PK_VARIANT(tbit(T_Q4_K) | tbit(T_Q5_K) | tbit(T_Q6_K) | tbit(T_Q8_0)),
    PK_VARIANT(tbit(T_Q4_0) | tbit(T_Q8_0)),
    PK_VARIANT(tbit(T_F32) | tbit(T_F16)),
    PK_VARIANT(FMT_ALL),
};
#undef PK_VARIANT

// Dynamic shared memory a phase kernel can use: the device's opt-in
// per-block maximum minus the kernels' static shared memory (queried once).
int smem_dynamic_max()
{
    static int v = 0;
    if (v == 0) {
        int dev = 0, optin = 0;
        cudaFuncAttributes fa;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            cudaFuncGetAttributes(&fa, phase_kernel<FMT_ALL>) != cudaSuccess) {
            cudaGetLastError();
            return SMEM_LIMIT - 4096;  // no device to ask: a conservative plan
        }
        v = optin - (int)fa.sharedSizeBytes;
    }
    return v;
}

// The first (smallest) variant that has every format in `need`.
static PhaseFn pick_variant(unsigned need)
{
    const int n = (int)(sizeof(VARIANTS) / sizeof(VARIANTS[0]));
    for (int i = 0; i < n; i++) {
        if ((need & ~VARIANTS[i].mask) == 0u) return VARIANTS[i].fn;
    }
    return VARIANTS[n - 1].fn;
}

// Formats a phase's matrices use.
static unsigned phase_formats(const Phase &p)
{
    unsigned need = 0u;
    if (p.kind != PH_MV) return need;
    for (int i = 0; i < p.nseg; i++) need |= tbit(p.seg[i].type);
    return need;
}

// finish_kernel for a tensor-parallel rank: the greedy token is the best of
// the ranks' argmax keys (each rank's logits phase published its key, as
// tagged words, to every rank's slots [world][4]).
__global__ void finish_kernel_tp(int *step, unsigned long long *amax, const uint64_t *keys, int world, int *tokens,
                                 int cap, int *err)
{
    const uint32_t tag = (uint32_t)step[4];
    unsigned long long best = 0ull;
    bool bad = false;
    for (int q = 0; q < world; q++) {
        uint32_t v[3];
        for (int i = 0; i < 3; i++) {
            const uint64_t *w = keys + (size_t)q * 4 + i;
            uint64_t x = ld_ll(w);
            const long long t0 = clock64();
            while (!ll_is(x, tag)) {
                if (aborted(err) || clock64() - t0 > LL_WAIT_LIMIT_CYCLES) {
                    atomicOr(err, ERR_TIMEOUT_WAIT);
                    break;
                }
                x = ld_ll(w);
            }
            v[i] = (uint32_t)x;
        }
        const unsigned long long k = ((unsigned long long)v[0] << 32) | v[1];
        if (k > best) best = k;
        if (v[2] != 0u) bad = true;
    }
    int tok = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    if (bad || best == 0ull) {
        tok = -1;
        atomicOr(err, ERR_NONFINITE);
    }
    const int n = step[2];
    if (n < cap) tokens[n] = tok;
    step[3] = tok;
    step[0] = tok < 0 ? 0 : tok;
    step[1] = step[1] + 1;
    step[2] = n + 1;
    step[4] = step[4] + 1;
    amax[0] = 0ull;
    amax[1] = 0ull;
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

// y = W x for F32 / F16 rows of any length, one warp per row, straight
// from global memory (the fallback when a row cannot be staged).
__global__ void mv_direct_kernel(const uint8_t *w, uint64_t rb, int type, int rows, int cols, const float *x,
                                 float *y)
{
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const uint8_t *row = w + (size_t)r * rb;
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) s = fmaf(decode_col(type, row, c), x[c], s);
    s = warp_sum(s);
    if (lane == 0) y[r] = s;
}

__global__ void fp16_table_kernel(float *out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < 65536) out[i] = h2f((uint32_t)i);
}

// ------------------------------------------------------------------ //
// Planning                                                           //
// ------------------------------------------------------------------ //

static int g_sm_count = 0;

static int sm_count()
{
    if (g_sm_count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (g_sm_count <= 0) g_sm_count = 1;
    }
    return g_sm_count;
}

// Rows per tile and tile numbering of a matvec phase, for `nw_total` warps
// and stages of at most `cap` bytes. even: tiles hold whole RoPE pairs. A
// one-matrix phase whose rows do not fit a stage streams each row in column
// chunks of whole quant blocks (one row per tile).
static void tile_phase(Phase &p, int nw_total, int cap, bool even)
{
    int total_rows = 0;
    for (int i = 0; i < p.nseg; i++) total_rows += p.seg[i].rows;
    const int r_par = (total_rows + nw_total - 1) / nw_total;
    p.nunits = (p.cols + 63) / 64;
    p.nchunk = 1;
    p.cunits = p.nunits;
    p.cbytes = 0;
    if (p.nseg == 1 && p.seg[0].rb + 32 > (uint64_t)cap) {
        const int type = p.seg[0].type, bw = block_weights(type), bb = block_bytes(type);
        // granule: the fewest whole units that are whole blocks
        const int gu = bw >= 64 ? bw / 64 : 1;
        const int gb = bw >= 64 ? bb : (64 / bw) * bb;
        int ng = (cap - 32 - 16) / gb;  // 16: a chunk may start off a 16-byte boundary
        if (ng < 1) ng = 1;
        p.cunits = ng * gu;
        p.cbytes = ng * gb;
        p.nchunk = (p.nunits + p.cunits - 1) / p.cunits;
    }
    int t = 0;
    for (int i = 0; i < p.nseg; i++) {
        MvSeg &s = p.seg[i];
        const int rcap = p.nchunk > 1 ? 1 : (int)((uint64_t)(cap - 32) / s.rb);
        int R = rcap < r_par ? rcap : r_par;
        if (even && (R & 1)) R = R + 1 <= rcap ? R + 1 : R - 1;  // whole RoPE pairs, within the stage
        if (R < (even ? 2 : 1)) R = even ? 2 : 1;
        if (R > RMAX) R = RMAX;
        s.R = R;
        s.tile0 = t;
        t += (s.rows + R - 1) / R;
    }
    p.ntiles = t;
}

// Bytes a stage needs to hold a tile (or a chunk) of the phase.
static int stage_need(const Phase &p)
{
    int need = 0;
    for (int i = 0; i < p.nseg; i++) {
        const MvSeg &s = p.seg[i];
        const uint64_t bytes = p.nchunk > 1 ? (uint64_t)p.cbytes + 16 : (uint64_t)s.R * s.rb;
        const int b = (int)((bytes + 32 + 15) / 16 * 16);  // bulk copies need 16-byte granularity
        if (b > need) need = b;
    }
    return need;
}

// Largest stage that leaves room for x in integer form (max_units units),
// the attention scratch and two stages per warp: at most 8 KB.
static int stage_cap(int max_units, int attn_floats)
{
    const int xq = (max_units * XQ_UNIT_BYTES + 127) / 128 * 128;
    int xs = xq + (max_units * 4 * XG_UNIT_WORDS + 127) / 128 * 128;
    const int at = (attn_floats * 4 + 127) / 128 * 128;
    if (at > xs) xs = at;
    const int bars = (DK_WARPS * 2 * 8 + 127) / 128 * 128;
    int cap = (smem_dynamic_max() - bars - xs) / (2 * DK_WARPS) / 16 * 16;
    if (cap > 8192) cap = 8192;
    return cap;
}

struct Layout {
    int warps, stages, stage_bytes, bar_bytes, xq_bytes, xs_bytes, attn_bytes;
    size_t smem;
};

// Shared-memory layout for phases with at most `max_units` 64-column units,
// stages of `stage` bytes and `attn_floats` of attention scratch.
static bool make_layout(Layout &L, int max_units, int stage, int attn_floats, int max_stages)
{
    L.xq_bytes = (max_units * XQ_UNIT_BYTES + 127) / 128 * 128;
    L.xs_bytes = L.xq_bytes + (max_units * 4 * XG_UNIT_WORDS + 127) / 128 * 128;
    L.attn_bytes = (attn_floats * 4 + 127) / 128 * 128;
    if (L.attn_bytes > L.xs_bytes) L.xs_bytes = L.attn_bytes;  // the two share one region
    L.stage_bytes = stage;
    for (L.warps = DK_WARPS; L.warps >= 1; L.warps /= 2) {
        for (L.stages = max_stages; L.stages >= 2; L.stages--) {
            L.bar_bytes = (L.warps * L.stages * 8 + 127) / 128 * 128;
            L.smem = (size_t)L.bar_bytes + L.xs_bytes + (size_t)L.warps * L.stages * stage;
            if (L.smem <= (size_t)smem_dynamic_max()) return true;
        }
    }
    return false;
}

static void fill_args(DecodeArgs &a, const Layout &L)
{
    a.stages = L.stages;
    a.stage_bytes = L.stage_bytes;
    a.bar_bytes = L.bar_bytes;
    a.xq_bytes = L.xq_bytes;
    a.xs_bytes = L.xs_bytes;
    a.attn_bytes = L.attn_bytes;
}

// Launch one phase as its own kernel on `st`.
static int launch_phase(const Phase &p, const int *step, int *err, cudaStream_t st, int grid_cap,
                        const float *rope_cs = nullptr, int rope_dim = 0, PhaseFn fn = nullptr, int seam = 0)
{
    if (fn == nullptr) fn = pick_variant(phase_formats(p));
    DecodeArgs a;
    memset(&a, 0, sizeof(a));
    a.one = p;
    a.one.cta0 = a.one.nct = 0;  // this launch's grid is the phase's alone
    a.phases = nullptr;
    a.nphases = 1;
    a.step = step;
    a.rope_cs = rope_cs;
    a.rope_dim = rope_dim;
    a.err = err;
    a.seam = seam;
    Layout L;
    const int attn_floats = p.kind == PH_ATTN ? attn_scratch_floats(p.hs, DK_WARPS) : 0;
    const int stage = p.kind == PH_MV ? stage_need(p) : 128;
    if (!make_layout(L, p.kind == PH_MV ? p.nunits : 1, stage, attn_floats, 3)) return 0;
    fill_args(a, L);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem) != cudaSuccess) {
        cudaGetLastError();  // a refused plan is not a context error
        return 0;
    }
    int grid = grid_cap;
    if (p.kind == PH_MV) {
        const int want = (p.ntiles + L.warps - 1) / L.warps;
        if (want < grid) grid = want;
    }
    if (grid < 1) grid = 1;
    if (p.epi == EPI_LOGITS && p.world > 1) {  // the CTAs of this launch that hold logits tiles
        a.one.ncta = 0;
        for (int b = 0; b < grid; b++) a.one.ncta += cta_has_tiles(p, b, L.warps, grid * L.warps) ? 1 : 0;
    }
    fn<<<grid, L.warps * 32, L.smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess;
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

// The seam's error words per device (DecodeArgs::seam: abort word,
// accumulated word, CTA count), allocated and zeroed on first use.
static int *device_err_word()
{
    static int *d_err[64] = {NULL};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NULL;
    if (d_err[dev] == NULL) {
        int *w = NULL;
        if (cudaMalloc(&w, 4 * sizeof(int)) != cudaSuccess) return NULL;
        if (cudaMemset(w, 0, 4 * sizeof(int)) != cudaSuccess) {
            cudaFree(w);
            return NULL;
        }
        d_err[dev] = w;
    }
    return d_err[dev];
}

extern "C" int gguf_cuda_matvec_error(void)
{
    int *w = device_err_word();
    if (w == NULL) return -1;
    int v = 0;
    if (cudaMemcpy(&v, w + 1, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v != 0 && cudaMemset(w + 1, 0, sizeof(int)) != cudaSuccess) return -1;
    return v != 0 ? 1 : 0;
}

extern "C" int gguf_cuda_matvec(const GGUFWeight *weight, const float *x, float *out, void *stream)
{
    if (!weight_ok(weight) || x == NULL || out == NULL || (const void *)x == (const void *)out) return 0;
    int *err = device_err_word();
    if (err == NULL) return 0;
    Phase p;
    memset(&p, 0, sizeof(p));
    p.kind = PH_MV;
    p.pro = PRO_PLAIN;
    p.epi = EPI_STORE;
    p.nseg = 1;
    p.seg[0].w = (const uint8_t *)weight->data;
    p.seg[0].rb = weight->row_bytes;
    p.seg[0].rows = (int)weight->rows;
    p.seg[0].type = (int)weight->type;
    p.cols = (int)weight->cols;
    p.xin = x;
    p.y = out;
    tile_phase(p, sm_count() * DK_WARPS, stage_cap((p.cols + 63) / 64, 0), false);
    Layout L;
    if (!make_layout(L, p.nunits, stage_need(p), 0, 3)) {
        if (weight->type != T_F32 && weight->type != T_F16) return 0;
        // Unquantized rows too long to stage: read them straight from HBM.
        const int rows = (int)weight->rows;
        mv_direct_kernel<<<(rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
            (const uint8_t *)weight->data, weight->row_bytes, (int)weight->type, rows, (int)weight->cols, x, out);
        return cudaGetLastError() == cudaSuccess;
    }
    return launch_phase(p, NULL, err, (cudaStream_t)stream, sm_count(), nullptr, 0, nullptr, 1);
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

// ------------------------------------------------------------------ //
// gguf_cuda_matvec_noalloc: the matvec with its scratch in device code //
// ------------------------------------------------------------------ //

// Scratch layout: [0, 256) header (words 0-2: the tile kernel's abort word,
// accumulated error word and CTA count, as DecodeArgs::seam describes),
// then the integer form of x for up to GGUF_CUDA_NOALLOC_MAX_COLS columns:
// digits (XQ_UNIT_BYTES per unit) at NA_Q_OFF, group info (XG_UNIT_WORDS
// words per unit) at NA_G_OFF - the layout stage_x writes to shared memory.
constexpr int NA_UNITS = GGUF_CUDA_NOALLOC_MAX_COLS / 64;
constexpr size_t NA_Q_OFF = 256;
constexpr size_t NA_G_OFF = NA_Q_OFF + (size_t)NA_UNITS * XQ_UNIT_BYTES;
constexpr size_t NA_SCRATCH_BYTES = NA_G_OFF + (size_t)NA_UNITS * XG_UNIT_WORDS * 4;
static_assert(NA_SCRATCH_BYTES == 184576, "scratch size is stated in gguf_cuda.h");
static_assert(NA_G_OFF % 16 == 0, "16-byte copies of the group info");

static __device__ __align__(256) uint8_t na_scratch[NA_SCRATCH_BYTES];

// One CTA: write x's integer form into the scratch (stage_x with global
// instead of shared destinations).
__global__ void __launch_bounds__(DK_WARPS * 32, 1) na_stage_kernel(const __grid_constant__ Phase p, uint8_t *scratch)
{
    stage_x(p, nullptr, scratch + NA_Q_OFF, reinterpret_cast<float *>(scratch + NA_G_OFF), 0u,
            reinterpret_cast<int *>(scratch));
}

// The matvec tiles of phase_kernel (same ring, same tiles, same row sums)
// with x's integer form copied from the scratch instead of staged per CTA.
__global__ void __launch_bounds__(DK_WARPS * 32, 1) na_matvec_kernel(const __grid_constant__ DecodeArgs a,
                                                                      const uint8_t *scratch)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const Phase &p = a.one;
    const int W = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * W + warp, NW = gridDim.x * W;

    Ring r;
    r.bars = reinterpret_cast<uint64_t *>(smem) + warp * a.stages;
    r.buf = smem + a.bar_bytes + a.xs_bytes + (size_t)warp * a.stages * a.stage_bytes;
    r.stages = a.stages;
    r.stage_bytes = a.stage_bytes;
    r.issued = r.consumed = 0;
    r.cp = r.ck = 0;
    uint8_t *xq = smem + a.bar_bytes;
    float *xg = reinterpret_cast<float *>(smem + a.bar_bytes + a.xq_bytes);

    if (lane == 0) {
        for (int s = 0; s < a.stages; s++) mbar_init(r.bars + s, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (lane == 0) ring_fill(r, &p, 1, gw, W, NW);

    const uint4 *sq = reinterpret_cast<const uint4 *>(scratch + NA_Q_OFF);
    const uint4 *sg = reinterpret_cast<const uint4 *>(scratch + NA_G_OFF);
    const int nq = p.nunits * XQ_UNIT_BYTES / 16, ng = p.nunits * XG_UNIT_WORDS * 4 / 16;
    for (int i = threadIdx.x; i < nq; i += blockDim.x) reinterpret_cast<uint4 *>(xq)[i] = __ldcg(sq + i);
    for (int i = threadIdx.x; i < ng; i += blockDim.x) reinterpret_cast<uint4 *>(xg)[i] = __ldcg(sg + i);
    __syncthreads();

    float racc = 0.0f;
    for (int k = 0;; k++) {
        const int t = tile_at(p, gw, W, NW, k / p.nchunk);
        if (t >= p.ntiles) break;
        const uint32_t slot = r.consumed % (uint32_t)a.stages;
        const uint32_t par = (r.consumed / (uint32_t)a.stages) & 1u;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait_or_abort(r.bars + slot, par, a.err));
        if (!ok) {
            if (lane == 0) atomicOr(a.err, ERR_TIMEOUT_MV);
        } else {
            run_tile<FMT_ALL>(p, t, k % p.nchunk, r.buf + slot * a.stage_bytes, xq, xg, 0, 0, nullptr, 0u, a.err,
                              lane, nullptr, racc, 1.0f);
        }
        __syncwarp();
        r.consumed++;
        if (lane == 0 && ok) ring_fill(r, &p, 1, gw, W, NW);
    }
    if (lane == 0 && r.issued != r.consumed) ring_drain(r);
    seam_finish(a.err);
}

static int na_fail(char *error, size_t cap, const char *msg)
{
    if (error != NULL && cap > 0) snprintf(error, cap, "%s", msg);
    return 0;
}

// Device address of the scratch, resolved once per device with that device
// current (cudaGetSymbolAddress allocates nothing; the array exists once
// the device code is loaded).
static uint8_t *na_scratch_addr(char *error, size_t cap)
{
    static uint8_t *addr[64] = {NULL};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        na_fail(error, cap, "gguf_cuda_matvec_noalloc: no current CUDA device.");
        return NULL;
    }
    if (addr[dev] == NULL) {
        void *p = NULL;
        const cudaError_t e = cudaGetSymbolAddress(&p, na_scratch);
        if (e != cudaSuccess || p == NULL) {
            if (error != NULL && cap > 0) {
                snprintf(error, cap, "gguf_cuda_matvec_noalloc: cudaGetSymbolAddress of the scratch failed on device %d: %s",
                         dev, cudaGetErrorString(e));
            }
            return NULL;
        }
        addr[dev] = (uint8_t *)p;
    }
    return addr[dev];
}

extern "C" int gguf_cuda_matvec_noalloc_error(void)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, na_scratch, sizeof(int), sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    if (v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(na_scratch, &zero, sizeof(int), sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
    }
    return v != 0 ? 1 : 0;
}

extern "C" int gguf_cuda_matvec_noalloc(const GGUFWeight *weight, const float *x, float *out, void *stream,
                                        char *error, size_t error_capacity)
{
    if (!weight_ok(weight) || x == NULL || out == NULL || (const void *)x == (const void *)out) {
        return na_fail(error, error_capacity,
                       "gguf_cuda_matvec_noalloc: invalid arguments (weight record, type, alignment, or x/out).");
    }
    if (weight->cols > (uint64_t)GGUF_CUDA_NOALLOC_MAX_COLS) {
        if (error != NULL && error_capacity > 0) {
            snprintf(error, error_capacity,
                     "gguf_cuda_matvec_noalloc: %llu columns exceed the scratch limit of %d "
                     "(GGUF_CUDA_NOALLOC_MAX_COLS); use gguf_cuda_matvec.",
                     (unsigned long long)weight->cols, GGUF_CUDA_NOALLOC_MAX_COLS);
        }
        return 0;
    }
    uint8_t *scratch = na_scratch_addr(error, error_capacity);
    if (scratch == NULL) return 0;
    cudaStream_t st = (cudaStream_t)stream;
    Phase p;
    memset(&p, 0, sizeof(p));
    p.kind = PH_MV;
    p.pro = PRO_PLAIN;
    p.epi = EPI_STORE;
    p.nseg = 1;
    p.seg[0].w = (const uint8_t *)weight->data;
    p.seg[0].rb = weight->row_bytes;
    p.seg[0].rows = (int)weight->rows;
    p.seg[0].type = (int)weight->type;
    p.cols = (int)weight->cols;
    p.xin = x;
    p.y = out;
    tile_phase(p, sm_count() * DK_WARPS, stage_cap((p.cols + 63) / 64, 0), false);  // gguf_cuda_matvec's tiles
    Layout L;
    if (!make_layout(L, p.nunits, stage_need(p), 0, 3)) {
        if (weight->type != T_F32 && weight->type != T_F16) {
            return na_fail(error, error_capacity, "gguf_cuda_matvec_noalloc: rows too long to stage.");
        }
        const int rows = (int)weight->rows;
        mv_direct_kernel<<<(rows + 7) / 8, 256, 0, st>>>((const uint8_t *)weight->data, weight->row_bytes,
                                                         (int)weight->type, rows, (int)weight->cols, x, out);
    } else {
        DecodeArgs a;
        memset(&a, 0, sizeof(a));
        a.one = p;
        a.nphases = 1;
        a.err = reinterpret_cast<int *>(scratch);
        fill_args(a, L);
        if (cudaFuncSetAttribute(na_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem) !=
            cudaSuccess) {
            cudaGetLastError();
            return na_fail(error, error_capacity, "gguf_cuda_matvec_noalloc: shared-memory plan rejected.");
        }
        int grid = (p.ntiles + L.warps - 1) / L.warps;
        if (grid > sm_count()) grid = sm_count();
        if (grid < 1) grid = 1;
        na_stage_kernel<<<1, DK_WARPS * 32, 0, st>>>(p, scratch);
        na_matvec_kernel<<<grid, L.warps * 32, L.smem, st>>>(a, scratch);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        if (error != NULL && error_capacity > 0) {
            snprintf(error, error_capacity, "gguf_cuda_matvec_noalloc: launch failed: %s", cudaGetErrorString(e));
        }
        return 0;
    }
    return 1;
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
    float *logits, *part, *norms, *rope_cs;
    void *kc, *vc;  // KV cache: float entries, or half with model.kv_half
    uint64_t *ll;  // tagged activations, per layer: q, k, v, attention out, x after Wo, gate and up, x after down
    int rope_dim;
    unsigned *count;
    int *step_d, *err_d, *tokens_d;
    int tokens_cap;
    unsigned long long *amax_d;
    Phase *phases_d;
    CopyEnt *copies_d;  // every warp's weight copies of a step (DecodeArgs::copies)
    int *copy_off_d;
    unsigned long long *trace_d;  // POCKET_CUDA_TRACE=1: per-phase end times of the last step
    cudaEvent_t ev0, ev1;
    // pinned host mirrors
    int *step_h;
    float *logits_h;
    int *err_h;
    int vocab, failed;
    // the step
    Phase *phases;  // host copy
    int nphases;
    Layout layout;
    int grid;
    PhaseFn fn;      // the phase_kernel variant for this model's formats
    int persistent;  // one cooperative launch per step (else one launch per phase)
    int use_graph;   // replay a captured graph (else launch directly)
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    // tensor parallel (tp.world > 1)
    PkdTp tp;
    uint64_t *peers[PKD_TP_MAX];  // each rank's exchange buffer (ll of that rank; peers[rank] = ll)
    int peer_mapped[PKD_TP_MAX];  // opened through IPC
    unsigned *lcount;             // logits CTAs finished
    // the model, kept for a build deferred to pkd_tp_connect
    PkdModel model;
    PkdTensor *tensors;           // 9 * n_layers, owned copies of the model's arrays
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
        // Two halves of the pinned staging buffer alternate: wait for the
        // copy that last used this half before refilling it.
        uint8_t *stg = (uint8_t *)c->staging + ((done / chunk) & 1) * chunk;
        if (done >= 2 * chunk && cuda_fail(c, cudaStreamSynchronize(c->stream), "upload sync", err, cap)) return 0;
        memcpy(stg, s + done, n);
        if (cuda_fail(c, cudaMemcpyAsync(c->arena + offset + done, stg, n, cudaMemcpyHostToDevice, c->stream),
                      "upload copy", err, cap))
            return 0;
        done += n;
    }
    return !cuda_fail(c, cudaStreamSynchronize(c->stream), "upload sync", err, cap);
}

static void seg_of(MvSeg &s, const PkdCtx *c, const PkdTensor &t, int kind)
{
    memset(&s, 0, sizeof(s));
    s.w = c->arena + t.offset;
    s.rb = t.row_bytes;
    s.rows = (int)t.rows;
    s.type = (int)t.type;
    s.kind = kind;
}

// Tagged activation words (offsets in words, each vector on a 256-byte
// boundary): per layer q, k, v, the attention output, the receive buffer
// of the Wo all-reduce, x after Wo, gate and up, the receive buffer of the
// down all-reduce, x after down; then the ranks' argmax slots and the
// logits (floats). The layout depends only on sizes common to all ranks, so
// it is the same on every rank of a tensor-parallel group (peers write into
// it at the same offsets).
struct LLPlan {
    size_t q, k, v, att, rwo, xmid, hb, rdn, xout, per_layer;
    size_t keys, logits, bx, bx_len, total;
};

static LLPlan ll_plan(const PkdModel *m)
{
    auto r32 = [](size_t n) { return (n + 31) / 32 * 32; };
    const PkdTp &t = m->tp;
    const size_t dim = (size_t)m->dim, hs = (size_t)m->head_size;
    const size_t qd = (size_t)t.q_heads * hs, kvd = (size_t)t.kv_heads * hs;
    const size_t recv = t.world > 1 ? r32((size_t)t.world * (size_t)t.own_max) : 0;
    LLPlan p;
    p.q = 0;
    p.k = p.q + r32(qd);
    p.v = p.k + r32(kvd);
    p.att = p.v + r32(kvd);
    p.rwo = p.att + r32(qd);
    p.xmid = p.rwo + recv;
    p.hb = p.xmid + r32(dim);
    p.rdn = p.hb + r32(2 * (size_t)t.hid_max);  // gate, then up
    p.xout = p.rdn + recv;
    p.per_layer = p.xout + r32(dim);
    p.keys = p.per_layer * (size_t)m->n_layers;
    p.logits = p.keys + r32(4 * (size_t)t.world);
    p.bx = p.logits + r32(((size_t)m->vocab_size + 1) / 2);
    // the batched step's exchanges (tensor parallel): per slot and rank up
    // to 64 rows of the residual stream or of the rank's vocabulary slice
    const size_t voc_max = ((size_t)m->vocab_size + (size_t)t.world - 1) / (size_t)t.world;
    p.bx_len = t.world > 1 ? r32(64 * (dim > voc_max ? dim : voc_max)) : 0;
    p.total = p.bx + 2 * (size_t)t.world * p.bx_len;
    return p;
}

// The phases of one decode step. Each phase's work starts where the
// previous phase's ended (tile rotation), so small phases do not all land
// on the first CTAs. A tensor-parallel rank computes its heads, hidden
// slice and vocabulary rows; Wo and down end in partial sums that an
// all-reduce phase combines (two per layer).
static int build_phases(PkdCtx *c, const PkdModel *m, int nw_total, int cap)
{
    const PkdTp &tp = m->tp;
    const int L = m->n_layers, dim = m->dim, hs = m->head_size, W = tp.world;
    const int kvd = hs * tp.kv_heads, qd = hs * tp.q_heads, km = tp.q_heads / tp.kv_heads;
    const int nsplit = attn_max_splits(tp.q_heads, c->grid, m->seq_len);
    const LLPlan lp = ll_plan(m);
    const int per = W > 1 ? 7 : 5;
    c->nphases = per * L + 1;
    c->phases = (Phase *)calloc((size_t)c->nphases, sizeof(Phase));
    if (c->phases == NULL) return 0;
    int acc = 0;  // the warp after the last tile of the previous phase
    auto rotate = [&](Phase &p) {
        p.off = acc;
        acc = (acc + p.ntiles) % nw_total;
    };
    // The QKV and Wo tiles avoid CTAs [0, heads), where the attention items
    // of one split each run: those CTAs start an attention item (its first
    // K/V tiles in flight) while the QKV rows are still being computed.
    const int heads = tp.q_heads;
    auto spare_attention_ctas = [&](Phase &p) {
        const int rest = c->grid - heads;
        if (rest >= 1 && rest * DK_WARPS >= p.ntiles) {
            p.cta0 = heads;
            p.nct = rest;
        }
    };
    auto tp_common = [&](Phase &p) {
        p.world = W;
        p.rank = tp.rank;
        p.own_max = tp.own_max;
        for (int q = 0; q < W; q++) {
            p.own0[q] = tp.own0[q];
            p.own[q] = tp.own[q];
        }
    };
    // all-reduce of the partials in recv (this rank's buffer) into `out`
    // (the same vector on every rank); residual `res` (null: the embedding row)
    auto all_reduce = [&](Phase &p, size_t recv, const uint64_t *res, size_t out) {
        p.kind = PH_AR;
        tp_common(p);
        p.off = (acc + DK_WARPS - 1) / DK_WARPS;
        p.xin_ll = c->ll + recv;
        p.res_ll = res;
        p.embd = c->arena + m->embd.offset;
        p.embd_rb = m->embd.row_bytes;
        p.embd_type = (int)m->embd.type;
        for (int q = 0; q < W; q++) p.peer[q] = c->peers[q] + out;
    };
    for (int l = 0; l < L; l++) {
        const size_t base = (size_t)l * lp.per_layer;
        uint64_t *ll = c->ll + base;
        const uint64_t *xin = l == 0 ? nullptr : c->ll + base - lp.per_layer + lp.xout;
        Phase *P = c->phases + per * l;
        Phase &qkv = P[0], &att = P[1], &wo = P[2];
        Phase &up = P[W > 1 ? 4 : 3], &dn = P[W > 1 ? 5 : 4];
        qkv.kind = PH_MV;
        qkv.pro = l == 0 ? PRO_EMBED_NORM : PRO_NORM;
        qkv.epi = EPI_QKV;
        qkv.nseg = 3;
        seg_of(qkv.seg[0], c, m->wq[l], KIND_Q);
        seg_of(qkv.seg[1], c, m->wk[l], KIND_K);
        seg_of(qkv.seg[2], c, m->wv[l], KIND_V);
        qkv.cols = dim;
        qkv.xin_ll = xin;
        qkv.norm = c->norms + (size_t)(2 * l) * dim;
        qkv.eps = m->rms_eps;
        qkv.embd = c->arena + m->embd.offset;
        qkv.embd_rb = m->embd.row_bytes;
        qkv.embd_type = (int)m->embd.type;
        qkv.q_ll = ll + lp.q;
        qkv.k_ll = ll + lp.k;
        qkv.v_ll = ll + lp.v;
        qkv.kc = c->kc;
        qkv.vc = c->vc;
        qkv.kv_half = m->kv_half;
        qkv.hs = hs;
        qkv.rope_dim = m->rope_dim;
        qkv.kv_dim = kvd;
        qkv.seq_len = m->seq_len;
        qkv.layer = l;
        tile_phase(qkv, nw_total, cap, true);
        spare_attention_ctas(qkv);
        rotate(qkv);

        att.kind = PH_ATTN;
        att.off = 0;  // head h's first split on CTA h, which has no QKV tiles
        att.aq_ll = ll + lp.q;
        att.ak_ll = ll + lp.k;
        att.av_ll = ll + lp.v;
        att.aout_ll = ll + lp.att;
        att.kc = c->kc;
        att.vc = c->vc;
        att.kv_half = m->kv_half;
        att.part = c->part;
        att.count = c->count + (size_t)l * tp.q_heads;
        att.layer = l;
        att.seq_len = m->seq_len;
        att.kv_dim = kvd;
        att.hs = hs;
        att.kv_mul = km;
        att.n_kv = tp.kv_heads;
        att.nsplit_max = nsplit;
        att.scale = m->att_scale;

        wo.kind = PH_MV;
        wo.pro = PRO_PLAIN;
        wo.nseg = 1;
        seg_of(wo.seg[0], c, m->wo[l], KIND_PLAIN);
        wo.cols = qd;
        wo.xin_ll = ll + lp.att;
        if (W > 1) {
            wo.epi = EPI_PEER;
            tp_common(wo);
            for (int q = 0; q < W; q++) wo.peer[q] = c->peers[q] + base + lp.rwo;
        } else {
            wo.epi = EPI_ADD;
            wo.res_ll = xin;  // null on layer 0: the embedding row
            wo.embd = c->arena + m->embd.offset;
            wo.embd_rb = m->embd.row_bytes;
            wo.embd_type = (int)m->embd.type;
            wo.y_ll = ll + lp.xmid;
        }
        tile_phase(wo, nw_total, cap, false);
        spare_attention_ctas(wo);
        rotate(wo);
        if (W > 1) all_reduce(P[3], base + lp.rwo, xin, base + lp.xmid);

        // gate and up as two row sets of one phase: gate rows to hb[0, hid);
        // an up row's epilogue takes its gate word and writes
        // silu(gate) * up to hb[hid, 2 hid), the down phase's input
        up.kind = PH_MV;
        up.pro = PRO_NORM;
        up.epi = EPI_STORE;
        up.nseg = 2;
        seg_of(up.seg[0], c, m->gate[l], KIND_PLAIN);
        seg_of(up.seg[1], c, m->up[l], KIND_UP);
        up.seg[1].yoff = m->hidden_dim;
        up.cols = dim;
        up.xin_ll = ll + lp.xmid;
        up.norm = c->norms + (size_t)(2 * l + 1) * dim;
        up.eps = m->rms_eps;
        up.y_ll = ll + lp.hb;
        tile_phase(up, nw_total, cap, false);
        rotate(up);

        dn.kind = PH_MV;
        dn.pro = PRO_PLAIN;
        dn.nseg = 1;
        seg_of(dn.seg[0], c, m->down[l], KIND_PLAIN);
        dn.cols = m->hidden_dim;
        dn.xin_ll = ll + lp.hb + m->hidden_dim;
        if (W > 1) {
            dn.epi = EPI_PEER;
            tp_common(dn);
            for (int q = 0; q < W; q++) dn.peer[q] = c->peers[q] + base + lp.rdn;
        } else {
            dn.epi = EPI_ADD;
            dn.res_ll = ll + lp.xmid;
            dn.y_ll = ll + lp.xout;
        }
        tile_phase(dn, nw_total, cap, false);
        rotate(dn);
        if (W > 1) all_reduce(P[6], base + lp.rdn, ll + lp.xmid, base + lp.xout);
    }
    Phase &lg = c->phases[per * L];
    lg.kind = PH_MV;
    lg.pro = PRO_NORM;
    lg.epi = EPI_LOGITS;
    lg.nseg = 1;
    seg_of(lg.seg[0], c, m->output, KIND_PLAIN);
    lg.cols = dim;
    lg.xin_ll = c->ll + (size_t)(L - 1) * lp.per_layer + lp.xout;
    lg.norm = c->norms + (size_t)(2 * L) * dim;
    lg.eps = m->rms_eps;
    lg.y = c->logits;
    lg.amax = c->amax_d;
    tile_phase(lg, nw_total, cap, false);
    rotate(lg);
    if (W > 1) {
        tp_common(lg);
        lg.voc0 = tp.voc0;
        for (int q = 0; q < W; q++) {
            lg.peer[q] = c->peers[q] + lp.logits;
            lg.keys[q] = c->peers[q] + lp.keys;
        }
        lg.done = c->lcount;
        for (int b = 0; b < c->grid; b++) lg.ncta += cta_has_tiles(lg, b, DK_WARPS, nw_total) ? 1 : 0;
    }
    return 1;
}

// Record one decode step on c->stream.
static int record_step(PkdCtx *c)
{
    cudaStream_t st = c->stream;
    if (c->persistent) {
        DecodeArgs a;
        memset(&a, 0, sizeof(a));
        a.phases = c->phases_d;
        a.nphases = c->nphases;
        a.copies = c->copies_d;
        a.copy_off = c->copy_off_d;
        a.step = c->step_d;
        a.rope_cs = c->rope_cs;
        a.rope_dim = c->rope_dim;
        a.err = c->err_d;
        a.trace = c->trace_d;
        fill_args(a, c->layout);
        cudaLaunchConfig_t cfg;
        memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(c->grid);
        cfg.blockDim = dim3(c->layout.warps * 32);
        cfg.dynamicSmemBytes = c->layout.smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, c->fn, a) != cudaSuccess) return 0;
    } else {
        // One launch per phase (the tagged words are complete by then).
        for (int i = 0; i < c->nphases; i++) {
            if (!launch_phase(c->phases[i], c->step_d, c->err_d, st, c->grid, c->rope_cs, c->rope_dim, c->fn)) {
                return 0;
            }
        }
    }
    if (c->tp.world > 1) {
        finish_kernel_tp<<<1, 1, 0, st>>>(c->step_d, c->amax_d, c->ll + ll_plan(&c->model).keys, c->tp.world,
                                          c->tokens_d, c->tokens_cap, c->err_d);
    } else {
        finish_kernel<<<1, 1, 0, st>>>(c->step_d, c->amax_d, c->tokens_d, c->tokens_cap, c->err_d);
    }
    return cudaGetLastError() == cudaSuccess;
}

static int env_flag(const char *name, int dflt)
{
    const char *v = getenv(name);
    return (v != NULL && *v) ? atoi(v) != 0 : dflt;
}

static int finalize(PkdCtx *c, char *err, size_t cap);

extern "C" int pkd_build(PkdCtx *c, const PkdModel *m, char *err, size_t cap)
{
    const size_t dim = (size_t)m->dim, hs = (size_t)m->head_size, kvd = hs * (size_t)m->n_kv_heads;
    const size_t cache = (size_t)m->n_layers * (size_t)m->seq_len * kvd * (m->kv_half ? 2 : 4);  // bytes
    const size_t nnorm = (2 * (size_t)m->n_layers + 1) * dim;
    if ((size_t)m->rope_dim > hs || hs % (m->kv_half ? 8 : 4) || hs > 256 || hs * (size_t)m->tp.q_heads > dim) {
        if (err && cap) snprintf(err, cap, "Unsupported model shape.");
        return 0;
    }
    cudaSetDevice(c->device);
    const int nsplit = attn_max_splits(m->n_heads, sm_count(), m->seq_len);
    const size_t part = (size_t)m->n_heads * nsplit * (hs + 2);
    const LLPlan lp = ll_plan(m);
    if (cuda_fail(c, cudaMalloc(&c->ll, lp.total * 8), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->kc, cache), "cudaMalloc(KV cache)", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->vc, cache), "cudaMalloc(KV cache)", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->part, part * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->norms, nnorm * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->rope_cs, (size_t)m->seq_len * m->rope_dim * 4 + 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->count, (size_t)m->n_layers * m->n_heads * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->lcount, 16), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->step_d, 32), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->err_d, 16), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->amax_d, 16), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaMalloc(&c->tokens_d, (size_t)m->seq_len * 4), "cudaMalloc", err, cap) ||
        cuda_fail(c, cudaEventCreate(&c->ev0), "cudaEventCreate", err, cap) ||
        cuda_fail(c, cudaEventCreate(&c->ev1), "cudaEventCreate", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->step_h, 32), "cudaMallocHost", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->logits_h, (size_t)m->vocab_size * 4), "cudaMallocHost", err, cap) ||
        cuda_fail(c, cudaMallocHost(&c->err_h, 16), "cudaMallocHost", err, cap)) {
        return 0;
    }
    c->logits = reinterpret_cast<float *>(c->ll + lp.logits);  // other ranks write their shards here
    c->vocab = m->vocab_size;
    c->tokens_cap = m->seq_len;
    c->tp = m->tp;
    c->peers[m->tp.rank] = c->ll;
    cudaStream_t st = c->stream;
    cudaMemsetAsync(c->kc, 0, cache, st);
    cudaMemsetAsync(c->vc, 0, cache, st);
    cudaMemsetAsync(c->count, 0, (size_t)m->n_layers * m->n_heads * 4, st);
    cudaMemsetAsync(c->lcount, 0, 16, st);
    cudaMemsetAsync(c->err_d, 0, 16, st);
    cudaMemsetAsync(c->amax_d, 0, 16, st);
    cudaMemsetAsync(c->ll, 0, lp.total * 8, st);  // tag 0: never a step's tag
    memset(c->step_h, 0, 32);
    c->step_h[4] = 1;  // the first step's tag
    cudaMemcpyAsync(c->step_d, c->step_h, 32, cudaMemcpyHostToDevice, st);
    c->rope_dim = m->rope_dim;
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
    // Keep the model description for the step (built now, or at connect).
    const int L = m->n_layers;
    c->tensors = (PkdTensor *)malloc(9 * (size_t)L * sizeof(PkdTensor));
    if (c->tensors == NULL) {
        if (err && cap) snprintf(err, cap, "Out of memory.");
        return 0;
    }
    const PkdTensor *src[9] = {m->wq, m->wk, m->wv, m->wo, m->gate, m->up, m->down, m->attn_norm, m->ffn_norm};
    for (int j = 0; j < 9; j++) memcpy(c->tensors + (size_t)j * L, src[j], (size_t)L * sizeof(PkdTensor));
    c->model = *m;
    c->model.wq = c->tensors;
    c->model.wk = c->tensors + L;
    c->model.wv = c->tensors + 2 * L;
    c->model.wo = c->tensors + 3 * L;
    c->model.gate = c->tensors + 4 * L;
    c->model.up = c->tensors + 5 * L;
    c->model.down = c->tensors + 6 * L;
    c->model.attn_norm = c->tensors + 7 * L;
    c->model.ffn_norm = c->tensors + 8 * L;
    c->model.rope_cs = nullptr;
    return m->tp.world > 1 ? 1 : finalize(c, err, cap);
}

extern "C" int pkd_tp_handle(PkdCtx *c, void *out64, char *err, size_t cap)
{
    if (c == NULL || out64 == NULL || c->tp.world < 2) return 0;
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    if (cuda_fail(c, cudaIpcGetMemHandle(&h, c->ll), "cudaIpcGetMemHandle", err, cap)) return 0;
    static_assert(sizeof(h) == 64, "exchange handles are 64 bytes");
    memcpy(out64, &h, 64);
    return 1;
}

extern "C" int pkd_tp_connect(PkdCtx *c, const void *handles, char *err, size_t cap)
{
    if (c == NULL || handles == NULL || c->tp.world < 2) return 0;
    cudaSetDevice(c->device);
    for (int q = 0; q < c->tp.world; q++) {
        if (q == c->tp.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + 64 * (size_t)q, 64);
        void *ptr = nullptr;
        if (cuda_fail(c, cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle",
                      err, cap))
            return 0;
        c->peers[q] = (uint64_t *)ptr;
        c->peer_mapped[q] = 1;
    }
    return finalize(c, err, cap);
}

// Every warp's weight copies for one decode step, in the order
// phase_kernel consumes its tiles (the MV phases in order; in each, tiles
// tile_at(p, gw, W, NW, k / nchunk) for k = 0, 1, ... below ntiles, chunk
// k % nchunk), uploaded for the rings' list refills. A CTA without tiles
// in a phase consumes nothing there, and neither does any of its warps.
static int build_copy_lists(PkdCtx *c, char *err, size_t cap)
{
    const int nw = c->grid * DK_WARPS;
    int *off = (int *)malloc(((size_t)nw + 1) * sizeof(int));
    if (off == NULL) {
        if (err && cap) snprintf(err, cap, "Out of memory.");
        return 0;
    }
    size_t total = 0;
    for (int pass = 0; pass < 2; pass++) {
        CopyEnt *ents = NULL;
        if (pass == 1) {
            ents = (CopyEnt *)malloc((total > 0 ? total : 1) * sizeof(CopyEnt));
            if (ents == NULL) {
                free(off);
                if (err && cap) snprintf(err, cap, "Out of memory.");
                return 0;
            }
        }
        size_t n = 0;
        for (int gw = 0; gw < nw; gw++) {
            off[gw] = (int)n;
            for (int pi = 0; pi < c->nphases; pi++) {
                const Phase &p = c->phases[pi];
                if (p.kind != PH_MV) continue;
                for (int k = 0;; k++) {
                    const int t = tile_at(p, gw, DK_WARPS, nw, k / p.nchunk);
                    if (t >= p.ntiles) break;
                    if (pass == 1) {
                        const Span sp = tile_span(p, t, k % p.nchunk);
                        ents[n].a0 = (uint64_t)sp.a0;
                        ents[n].bulk = sp.bulk;
                        ents[n].tail = sp.tail;
                    }
                    n++;
                }
            }
        }
        off[nw] = (int)n;
        total = n;
        if (pass == 1) {
            const int ok = !cuda_fail(c, cudaMalloc(&c->copies_d, (total > 0 ? total : 1) * sizeof(CopyEnt)),
                                      "cudaMalloc", err, cap) &&
                           !cuda_fail(c, cudaMalloc(&c->copy_off_d, ((size_t)nw + 1) * sizeof(int)), "cudaMalloc",
                                      err, cap) &&
                           !cuda_fail(c, cudaMemcpy(c->copies_d, ents, total * sizeof(CopyEnt),
                                                    cudaMemcpyHostToDevice), "copy list upload", err, cap) &&
                           !cuda_fail(c, cudaMemcpy(c->copy_off_d, off, ((size_t)nw + 1) * sizeof(int),
                                                    cudaMemcpyHostToDevice), "copy list upload", err, cap);
            free(ents);
            free(off);
            return ok;
        }
    }
    free(off);
    return 0;
}

// Phases, shared-memory plan, kernel variant and the captured step.
static int finalize(PkdCtx *c, char *err, size_t cap)
{
    const PkdModel *m = &c->model;
    cudaStream_t st = c->stream;
    c->persistent = env_flag("POCKET_CUDA_PERSISTENT", 1);
    c->use_graph = !env_flag("POCKET_CUDA_EAGER", 0);
    c->grid = sm_count();
    // stages as large as the shared memory left after x and the attention
    // scratch allows (rows longer than a stage go in column chunks)
    const int widest = m->dim > m->hidden_dim ? m->dim : m->hidden_dim;
    const int scap = stage_cap((widest + 63) / 64, attn_scratch_floats(m->head_size, DK_WARPS));
    if (!build_phases(c, m, c->grid * DK_WARPS, scap)) {
        if (err && cap) snprintf(err, cap, "Out of memory.");
        return 0;
    }
    if (env_flag("POCKET_CUDA_TRACE", 0) &&
        cuda_fail(c, cudaMalloc(&c->trace_d, (size_t)(3 * c->nphases + 1 + 2 * c->grid * c->nphases) * 8), "cudaMalloc", err, cap)) {
        return 0;
    }
    // Failure-injection hook for tests: POCKET_CUDA_TEST_STALL=<phase>:<us>
    // makes phase <phase>'s input polls wait for a tag that is never
    // written, giving up after <us> microseconds (at 2 GHz), so that the
    // step ends with a timed-out wait and the handle reports it.
    const char *stall = getenv("POCKET_CUDA_TEST_STALL");
    if (stall != NULL && *stall) {
        int ph = -1;
        long long us = 0;
        if (sscanf(stall, "%d:%lld", &ph, &us) == 2 && ph >= 0 && ph < c->nphases && us > 0 &&
            c->phases[ph].kind == PH_MV) {
            c->phases[ph].stall = us * 2000;
        }
    }
    unsigned need = 0u;
    for (int i = 0; i < c->nphases; i++) need |= phase_formats(c->phases[i]);
    c->fn = pick_variant(need);
    int max_units = 1, stage = 128;
    for (int i = 0; i < c->nphases; i++) {
        if (c->phases[i].kind != PH_MV) continue;
        if (c->phases[i].nunits > max_units) max_units = c->phases[i].nunits;
        const int need = stage_need(c->phases[i]);
        if (need > stage) stage = need;
    }
    const int attn_floats = attn_scratch_floats(m->head_size, DK_WARPS);
    if (!make_layout(c->layout, max_units, stage, attn_floats, 4)) {
        if (err && cap) snprintf(err, cap, "Model rows or context too large for the shared-memory plan.");
        return 0;
    }
    if (c->persistent) {
        int per_sm = 0;
        if (c->layout.warps != DK_WARPS ||  // tiles were numbered for DK_WARPS warps per CTA
            cudaFuncSetAttribute(c->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->layout.smem) !=
                cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, c->fn, c->layout.warps * 32,
                                                          c->layout.smem) != cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            c->persistent = 0;  // no co-residency guarantee: one launch per phase instead
        }
    }
    if (cuda_fail(c, cudaMalloc(&c->phases_d, (size_t)c->nphases * sizeof(Phase)), "cudaMalloc", err, cap) ||
        cuda_fail(c,
                  cudaMemcpyAsync(c->phases_d, c->phases, (size_t)c->nphases * sizeof(Phase),
                                  cudaMemcpyHostToDevice, st),
                  "phase upload", err, cap) ||
        !build_copy_lists(c, err, cap) ||
        cuda_fail(c, cudaStreamSynchronize(st), "build sync", err, cap)) {
        return 0;
    }
    if (!c->use_graph) return 1;
    // Capture one decode step as a graph; replays read token/pos from step_d.
    // If the cooperative launch cannot be captured, capture the per-phase
    // launches instead.
    for (int attempt = 0; attempt < 2; attempt++) {
        if (cuda_fail(c, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "capture", err, cap)) {
            return 0;
        }
        const int ok = record_step(c);
        cudaError_t e = cudaStreamEndCapture(st, &c->graph);
        if (ok && e == cudaSuccess && cudaGraphInstantiate(&c->exec, c->graph, 0) == cudaSuccess) return 1;
        cudaGetLastError();
        if (c->graph) {
            cudaGraphDestroy(c->graph);
            c->graph = NULL;
        }
        if (!c->persistent) {
            if (err && cap) snprintf(err, cap, "Cannot record the decode step (%s).", cudaGetErrorString(e));
            return 0;
        }
        c->persistent = 0;
    }
    return 0;
}

static int launch_step(PkdCtx *c)
{
    if (c->use_graph) return cudaGraphLaunch(c->exec, c->stream) == cudaSuccess;
    return record_step(c);
}

static int run_step(PkdCtx *c, int token, int pos, int want_logits)
{
    if (c == NULL || c->failed) return 0;
    c->step_h[0] = token;
    c->step_h[1] = pos;
    c->step_h[2] = 0;
    cudaStream_t st = c->stream;
    cudaMemcpyAsync(c->step_d, c->step_h, 12, cudaMemcpyHostToDevice, st);
    launch_step(c);
    if (want_logits) cudaMemcpyAsync(c->logits_h, c->logits, (size_t)c->vocab * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(c->step_h, c->step_d, 16, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(c->err_h, c->err_d, 4, cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        snprintf(c->msg, sizeof(c->msg), "decode step: %s", cudaGetErrorString(e));
        c->failed = 1;
        return 0;
    }
    if (c->err_h[0] & ERR_NONFINITE) cudaMemsetAsync(c->err_d, 0, 4, st);  // a value, not a failure
    if (c->err_h[0] & ERR_FATAL) {
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
    return c->step_h[3];  // the finish kernel's token, -1 for a non-finite logit
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
    for (int i = 0; i < n; i++) launch_step(c);
    cudaEventRecord(c->ev1, st);
    if (n > 0) cudaMemcpyAsync(out, c->tokens_d, (size_t)n * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(c->err_h, c->err_d, 4, cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        snprintf(c->msg, sizeof(c->msg), "generate: %s", cudaGetErrorString(e));
        c->failed = 1;
        return 0;
    }
    if (c->err_h[0] & ERR_FATAL) {
        snprintf(c->msg, sizeof(c->msg), "generate: device wait timed out (code %d)", c->err_h[0]);
        c->failed = 1;
        return 0;
    }
    if (c->err_h[0] & ERR_NONFINITE) cudaMemsetAsync(c->err_d, 0, 4, st);  // reported per token as -1
    if (device_ms != NULL) cudaEventElapsedTime(device_ms, c->ev0, c->ev1);
    return 1;
}

extern "C" int pkd_trace(PkdCtx *c, unsigned long long *out, int cap)
{
    if (c == NULL || c->trace_d == NULL || out == NULL) return 0;
    const int all = 3 * c->nphases + 1 + 2 * c->grid * c->nphases;
    const int n = all < cap ? all : cap;
    if (cudaMemcpy(out, c->trace_d, (size_t)n * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    return n;
}

extern "C" int pkd_kv_write(PkdCtx *c, int layer, int pos0, int npos, const float *k, const float *v, char *err,
                            size_t cap)
{
    if (c == NULL || c->kc == NULL || k == NULL || v == NULL) return 0;
    const PkdModel &m = c->model;
    if (layer < 0 || layer >= m.n_layers || pos0 < 0 || npos < 0 || pos0 > m.seq_len - npos) {
        if (err && cap) snprintf(err, cap, "KV write outside the cache.");
        return 0;
    }
    cudaSetDevice(c->device);
    const size_t kvd = (size_t)m.head_size * (size_t)m.tp.kv_heads;
    const size_t off = ((size_t)layer * (size_t)m.seq_len + (size_t)pos0) * kvd, n = (size_t)npos * kvd;
    return !cuda_fail(c, kv_upload(c->kc, m.kv_half, off, k, n, c->stream), "KV write", err, cap) &&
           !cuda_fail(c, kv_upload(c->vc, m.kv_half, off, v, n, c->stream), "KV write", err, cap);
}

extern "C" const char *pkd_error(const PkdCtx *c)
{
    return c ? c->msg : "";
}

extern "C" int pkd_view(PkdCtx *c, PkdView *out)
{
    if (c == NULL || out == NULL || c->tensors == NULL || c->norms == NULL) return 0;
    memset(out, 0, sizeof(*out));
    out->rank = c->tp.world > 1 ? c->tp.rank : 0;
    out->world = c->tp.world > 1 ? c->tp.world : 1;
    if (out->world > 1) {
        for (int q = 0; q < out->world; q++) {
            if (c->peers[q] == NULL) return 0;  // not connected yet
            out->peers[q] = c->peers[q];
        }
        const LLPlan lp = ll_plan(&c->model);
        out->bx = lp.bx;
        out->bx_len = lp.bx_len;
    }
    out->device = c->device;
    out->stream = (void *)c->stream;
    out->arena = c->arena;
    out->norms = c->norms;
    out->rope_cs = c->rope_cs;
    out->model = &c->model;
    out->kc = c->kc;
    out->vc = c->vc;
    return 1;
}

extern "C" int pkd_launches_per_step(const PkdCtx *c)
{
    if (c == NULL) return 0;
    return c->persistent ? 2 : c->nphases + 1;
}

extern "C" void pkd_destroy(PkdCtx *c)
{
    if (c == NULL) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->exec) cudaGraphExecDestroy(c->exec);
    if (c->graph) cudaGraphDestroy(c->graph);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    for (int q = 0; q < PKD_TP_MAX; q++) {
        if (c->peer_mapped[q]) cudaIpcCloseMemHandle(c->peers[q]);
    }
    free(c->tensors);
    void *dev[] = {c->arena, c->ll, c->lcount, c->kc, c->vc, c->part, c->norms,
                   c->rope_cs, c->count, c->step_d, c->err_d, c->amax_d, c->tokens_d, c->phases_d,
                   c->copies_d, c->copy_off_d,
                   c->trace_d};
    for (size_t i = 0; i < sizeof(dev) / sizeof(dev[0]); i++) {
        if (dev[i]) cudaFree(dev[i]);
    }
    void *host[] = {c->staging, c->step_h, c->logits_h, c->err_h};
    for (size_t i = 0; i < sizeof(host) / sizeof(host[0]); i++) {
        if (host[i]) cudaFreeHost(host[i]);
    }
    if (c->stream) cudaStreamDestroy(c->stream);
    free(c->phases);
    free(c);
}
