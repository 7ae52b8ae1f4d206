// pk_stream.cuh - the phase executor shared by every kernel of the decode
// path: one "phase" is a fused dequant-matvec over up to three matrices
// (with its prologue and epilogue) or the attention of one layer.
//
// Data movement. Every warp owns a ring of shared-memory stages and an
// mbarrier per stage. Lane 0 issues 1-D bulk copies (cp.async.bulk, the
// TMA engine) of whole packed rows into the ring; the tiles a warp will
// consume are known in advance for every phase, so in the persistent decode
// kernel the ring keeps streaming the NEXT phases' weights while the warp
// waits for its inputs. Weights never depend on activations.
//
// Compute. x is staged once per phase and CTA in integer form (pk_quant.cuh);
// each lane owns 64-column units; a row's units are summed over the warp.
//
// Hand-offs. Activations that one phase produces and the next consumes are
// "tagged words" (the scheme of NCCL's LL protocol): one 64-bit word per
// value, the step's tag in the high half and the float in the low half,
// stored and loaded as single 64-bit accesses. A consumer polls exactly the
// words it needs until they carry the current step's tag, so there is no
// grid-wide barrier between phases: a phase starts in a CTA as soon as its
// own inputs have landed, and a CTA with no work in a phase skips it.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "pk_quant.cuh"

namespace pk {

constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;  // ~2 s at 2 GHz
// Tagged words may come from another GPU whose step started later (ranks
// launch independently): a longer bound.
constexpr long long LL_WAIT_LIMIT_CYCLES = 20000000000LL;  // ~10 s at 2 GHz
// A poll checks the abort flag (one more global load) only once it has
// been failing this long (~10 us), so that a normal short wait costs one
// round trip per retry.
constexpr long long LL_ABORT_CHECK_CYCLES = 20000LL;
constexpr int TP_MAX = 8;  // ranks of a tensor-parallel group

enum { PH_MV = 0, PH_ATTN = 1, PH_AR = 2 };
// PRO_SWIGLU stages silu(gate) * up from a gate|up vector; the decode step's
// down phase no longer uses it (its up rows' epilogue, KIND_UP, writes the
// product), the prologue stays for phases built on a gate|up input.
enum { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED_NORM = 2, PRO_SWIGLU = 3 };
enum { EPI_STORE = 0, EPI_ADD = 1, EPI_QKV = 2, EPI_LOGITS = 4, EPI_PEER = 5 };
enum { KIND_PLAIN = 0, KIND_Q = 1, KIND_K = 2, KIND_V = 3, KIND_UP = 4 };
enum { ERR_TIMEOUT_MV = 1, ERR_TIMEOUT_WAIT = 2, ERR_NONFINITE = 4 };
constexpr int ERR_FATAL = ERR_TIMEOUT_MV | ERR_TIMEOUT_WAIT;

// ------------------------------------------------------------------ //
// PTX helpers                                                        //
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

__device__ __forceinline__ bool aborted(const int *err);

// mbar_wait_bounded that also gives up when another thread has recorded a
// timeout (checked only after ~10 us of waiting, so neither a ready stage
// nor a short wait costs a global load).
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity, const int *err)
{
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (clock64() - t0 < 20000LL) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    if (aborted(err)) return false;
    return mbar_wait_bounded(bar, parity);
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool aborted(const int *err)
{
    return (*(volatile const int *)err & ERR_FATAL) != 0;
}

// ------------------------------------------------------------------ //
// Tagged words                                                       //
// ------------------------------------------------------------------ //

__device__ __forceinline__ void st_ll(uint64_t *p, float v, uint32_t tag)
{
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// The same, for words another GPU reads (system scope).
__device__ __forceinline__ void st_ll_sys(uint64_t *p, float v, uint32_t tag)
{
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ void st_u64_sys(uint64_t *p, uint64_t w)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_ll(const uint64_t *p)
{
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Two words from a 16-byte aligned address (each one a single access).
__device__ __forceinline__ void ld_ll2(const uint64_t *p, uint64_t &a, uint64_t &b)
{
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ bool ll_is(uint64_t w, uint32_t tag)
{
    return (uint32_t)(w >> 32) == tag;
}

__device__ __forceinline__ float ll_val(uint64_t w)
{
    return __uint_as_float((uint32_t)w);
}

// Value of the tagged word at p once it carries `tag` (bounded wait; on a
// timeout the error word is set and whatever is there is returned).
__device__ __forceinline__ float ll_read(const uint64_t *p, uint32_t tag, int *err)
{
    uint64_t w = ld_ll(p);
    if (ll_is(w, tag)) return ll_val(w);
    const long long t0 = clock64();
    do {
        w = ld_ll(p);
        if (ll_is(w, tag)) break;
        const long long dt = clock64() - t0;
        if (dt > LL_ABORT_CHECK_CYCLES && aborted(err)) break;
        if (dt > LL_WAIT_LIMIT_CYCLES) {
            atomicOr(err, ERR_TIMEOUT_WAIT);
            break;
        }
    } while (true);
    return ll_val(w);
}

// Values of n (<= 8) tagged words at each of pa and pb (64-byte aligned
// when n == 8), polled together so that both wait in one round trip per
// retry; va/vb[e] = 0 for e >= n. Bounded as ll_read.
__device__ __forceinline__ void ll_read8x2(const uint64_t *pa, const uint64_t *pb, int n, uint32_t tag, float *va,
                                           float *vb, int *err, long long limit = LL_WAIT_LIMIT_CYCLES)
{
    uint64_t w[16];
    long long t0 = 0;
    bool first = true;
    for (;;) {
        if (n >= 8) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                ld_ll2(pa + 2 * k, w[2 * k], w[2 * k + 1]);
                ld_ll2(pb + 2 * k, w[8 + 2 * k], w[8 + 2 * k + 1]);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                w[e] = e < n ? ld_ll(pa + e) : ((uint64_t)tag << 32);
                w[8 + e] = e < n ? ld_ll(pb + e) : ((uint64_t)tag << 32);
            }
        }
        bool ok = true;
#pragma unroll
        for (int e = 0; e < 16; e++) ok = ok && ll_is(w[e], tag);
        if (ok) break;
        if (first) {
            t0 = clock64();
            first = false;
        } else {
            const long long dt = clock64() - t0;
            if (dt > LL_ABORT_CHECK_CYCLES && aborted(err)) break;
            if (dt > limit) {
                atomicOr(err, ERR_TIMEOUT_WAIT);
                break;
            }
        }
    }
#pragma unroll
    for (int e = 0; e < 8; e++) {
        va[e] = e < n ? ll_val(w[e]) : 0.0f;
        vb[e] = e < n ? ll_val(w[8 + e]) : 0.0f;
    }
}

// Values of the n (<= 8) tagged words at p (64-byte aligned when n == 8),
// waiting (bounded) until all carry `tag`; v[e] = 0 for e >= n.
__device__ __forceinline__ void ll_read8(const uint64_t *p, int n, uint32_t tag, float *v, int *err,
                                         long long limit = LL_WAIT_LIMIT_CYCLES)
{
    uint64_t w[8];
    long long t0 = 0;
    bool first = true;
    for (;;) {
        if (n >= 8) {
#pragma unroll
            for (int k = 0; k < 4; k++) ld_ll2(p + 2 * k, w[2 * k], w[2 * k + 1]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) w[e] = e < n ? ld_ll(p + e) : ((uint64_t)tag << 32);
        }
        bool ok = true;
#pragma unroll
        for (int e = 0; e < 8; e++) ok = ok && ll_is(w[e], tag);
        if (ok) break;
        if (first) {
            t0 = clock64();
            first = false;
        } else {
            const long long dt = clock64() - t0;
            if (dt > LL_ABORT_CHECK_CYCLES && aborted(err)) break;
            if (dt > limit) {
                atomicOr(err, ERR_TIMEOUT_WAIT);
                break;
            }
        }
    }
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = e < n ? ll_val(w[e]) : 0.0f;
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
// Phase description                                                  //
// ------------------------------------------------------------------ //

struct MvSeg {
    const uint8_t *w;  // row 0 of the matrix
    uint64_t rb;       // bytes per row
    int rows, type, R, tile0, kind;
    int yoff;          // EPI_STORE: row r goes to output element yoff + r
};

// 16-byte multiple: the decode step bulk-copies each phase's descriptor
// into shared memory.
struct alignas(16) Phase {
    int kind, pro, epi;
    long long stall;      // test hook, normally 0: > 0 makes this phase's input polls wait for
                          // a tag no producer writes, giving up after `stall` cycles
    int off;              // work rotation: tile t goes to warp slot (t + off) % slots,
                          // attention item i to CTA (i + off) % CTAs
    int cta0, nct;        // the tiles go to the warps of CTAs [cta0, cta0 + nct) (mod the
                          // grid; nct 0: every CTA), warp-major: warp 0 of each CTA first
    // fused matvec
    MvSeg seg[3];
    int nseg, ntiles, cols, nunits;
    int nchunk, cunits, cbytes;  // rows longer than a stage: nchunk column chunks of cunits
                                 // 64-column units (cbytes bytes), one row per tile
    const float *xin;         // input vector as floats (device seam), or
    const uint64_t *xin_ll;   // as tagged words (decode step)
    const float *norm;        // RMSNorm weights (PRO_NORM / PRO_EMBED_NORM); PRO_SWIGLU
                              //   reads gate at xin_ll[c] and up at xin_ll[cols + c]
    float eps;
    float *y;                 // float output (EPI_STORE of the seam, EPI_LOGITS)
    uint64_t *y_ll;           // tagged output (EPI_STORE / EPI_ADD)
    const uint64_t *res_ll;   // EPI_ADD residual (null: the embedding row)
    const uint8_t *embd;      // embedding table, row bytes, type (PRO_EMBED_NORM,
    uint64_t embd_rb;         //   and the residual of layer 0's EPI_ADD)
    int embd_type;
    uint64_t *q_ll, *k_ll, *v_ll;  // EPI_QKV outputs (tagged)
    void *kc, *vc;                 // KV cache (EPI_QKV appends, attention reads):
    int kv_half;                   //   float entries, or IEEE half when kv_half
    int hs, rope_dim, kv_dim, seq_len, layer;
    unsigned long long *amax;  // EPI_LOGITS: [0] packed argmax, [1] non-finite flag
    // attention
    const uint64_t *aq_ll, *ak_ll, *av_ll;  // q, and this position's k, v
    uint64_t *aout_ll;
    float *part;
    unsigned *count;
    int kv_mul, n_kv, nsplit_max;
    float scale;
    // tensor parallel (world > 1)
    int world, rank, own_max;
    int own0[TP_MAX], own[TP_MAX];  // rank q reduces elements [own0[q], own0[q] + own[q])
    uint64_t *peer[TP_MAX];   // EPI_PEER: each rank's receive buffer [world][own_max];
                              // PH_AR: each rank's output vector; EPI_LOGITS: each rank's logits
    uint64_t *keys[TP_MAX];   // EPI_LOGITS: each rank's argmax slots [world][4]
    int voc0;                 // EPI_LOGITS: vocabulary row of local row 0
    unsigned *done;           // EPI_LOGITS: CTAs finished; the last publishes the argmax
    int ncta;                 // EPI_LOGITS: CTAs with logits tiles
};

constexpr int NO_TILE = 0x7FFFFFFF;

// Slot of warp gw (W warps per CTA, nw in the grid) among the phase's
// warps, or -1 when its CTA takes no tiles. Slots run warp-major over the
// phase's CTAs (warp 0 of every CTA, then warp 1, ...), so that a phase
// with fewer tiles than warps still spreads over all of its SMs.
__host__ __device__ inline int warp_slot(const Phase &p, int gw, int W, int nw, int &nslots)
{
    const int G = nw / W, b = gw / W, w = gw % W;
    const int nct = p.nct > 0 && p.nct < G ? p.nct : G;
    nslots = nct * W;
    const int lb = ((b - p.cta0) % G + G) % G;
    return lb < nct ? w * nct + lb : -1;
}

// Tile k (0, 1, ...) of warp gw among nw warps, W per CTA (>= ntiles: none).
__host__ __device__ inline int tile_at(const Phase &p, int gw, int W, int nw, int k)
{
    int ns = 1;
    const int s0 = warp_slot(p, gw, W, nw, ns);
    if (s0 < 0) return NO_TILE;
    return (s0 + ns - p.off % ns) % ns + k * ns;
}

// Does any of the W warps of CTA b own a tile of p?
__host__ __device__ inline bool cta_has_tiles(const Phase &p, int b, int W, int nw)
{
    if (p.ntiles <= 0) return false;
    for (int w = 0; w < W; w++) {
        if (tile_at(p, b * W + w, W, nw, 0) < p.ntiles) return true;
    }
    return false;
}

// ------------------------------------------------------------------ //
// Bulk-copy ring                                                     //
// ------------------------------------------------------------------ //

struct Span {
    uintptr_t a0;
    uint32_t bulk, tail;
};

// Bytes [st, st + n) land at buf + (st & 15): the 16-byte aligned body via
// the bulk-copy engine, the sub-16-byte tail (only a matrix's last row can
// end unaligned) via plain loads, so nothing past the matrix is read.
__host__ __device__ inline Span make_span(uintptr_t st, uint64_t n)
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

__host__ __device__ inline const MvSeg &find_seg(const Phase &p, int t)
{
    if (p.nseg > 2 && t >= p.seg[2].tile0) return p.seg[2];
    if (p.nseg > 1 && t >= p.seg[1].tile0) return p.seg[1];
    return p.seg[0];
}

// Bytes of chunk `chunk` of tile t of phase p in global memory, as
// issue_tile copies them (host and device).
__host__ __device__ inline Span tile_span(const Phase &p, int t, int chunk)
{
    const MvSeg &s = find_seg(p, t);
    const int r0 = (t - s.tile0) * s.R;
    const int nr = s.R < s.rows - r0 ? s.R : s.rows - r0;
    uintptr_t st = reinterpret_cast<uintptr_t>(s.w) + (uintptr_t)r0 * s.rb;
    uint64_t n = (uint64_t)nr * s.rb;
    if (p.nchunk > 1) {  // one row, one chunk of it
        const uint64_t off = (uint64_t)chunk * (uint64_t)p.cbytes;
        st += off;
        n = s.rb - off < (uint64_t)p.cbytes ? s.rb - off : (uint64_t)p.cbytes;
    }
    return make_span(st, n);
}

// Lane 0: issue the copies of chunk `chunk` of tile t of phase p into buf;
// completes on bar.
__device__ __forceinline__ void issue_tile(const Phase &p, int t, int chunk, uint8_t *buf, uint64_t *bar)
{
    const Span sa = tile_span(p, t, chunk);
    mbar_expect_tx(bar, sa.bulk);
    fill_span(sa, buf, bar);
}

// One entry of a warp's copy list: the span of one tile (or chunk) it
// consumes, in consumption order. 16 bytes, read with one vector load.
struct CopyEnt {
    uint64_t a0;
    uint32_t bulk, tail;
};

__device__ __forceinline__ CopyEnt ld_copy(const CopyEnt *p)
{
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
    CopyEnt e;
    e.a0 = ((uint64_t)v.y << 32) | v.x;
    e.bulk = v.z;
    e.tail = v.w;
    return e;
}

// A warp's ring and its producer cursor: (phase index, tile ordinal) when
// it walks the phase descriptors, or the position in its copy list.
struct Ring {
    uint64_t *bars;
    uint8_t *buf;
    int stages, stage_bytes;
    uint32_t issued, consumed;
    int cp, ck;
    const CopyEnt *list;  // null: walk the descriptors
    uint32_t nlist, next;
    CopyEnt pre;          // list[next], loaded one refill ahead
};

// Lane 0: top the ring up with this warp's next tiles, in consumption order,
// across phase boundaries.
__device__ __forceinline__ void ring_fill(Ring &r, const Phase *ph, int nph, int gw, int W, int nw_total)
{
    while (r.issued - r.consumed < (uint32_t)r.stages && r.cp < nph) {
        const Phase &p = ph[r.cp];
        const int t = p.kind == PH_MV ? tile_at(p, gw, W, nw_total, r.ck / p.nchunk) : 0;
        if (p.kind != PH_MV || t >= p.ntiles) {
            r.cp++;
            r.ck = 0;
            continue;
        }
        const uint32_t slot = r.issued % (uint32_t)r.stages;
        issue_tile(p, t, r.ck % p.nchunk, r.buf + slot * r.stage_bytes, r.bars + slot);
        r.issued++;
        r.ck++;
    }
}

// Lane 0: ring_fill from the warp's copy list (built on the host in the
// order the warp consumes its tiles). A refill issues from registers: the
// entry after the one issued is loaded at once, and that load completes
// while the warp computes, instead of the descriptor walk's dependent L2
// round trips at the end of every phase.
__device__ __forceinline__ void ring_fill_list(Ring &r)
{
    while (r.issued - r.consumed < (uint32_t)r.stages && r.next < r.nlist) {
        const uint32_t slot = r.issued % (uint32_t)r.stages;
        Span sa;
        sa.a0 = (uintptr_t)r.pre.a0;
        sa.bulk = r.pre.bulk;
        sa.tail = r.pre.tail;
        mbar_expect_tx(r.bars + slot, sa.bulk);
        fill_span(sa, r.buf + slot * r.stage_bytes, r.bars + slot);
        r.issued++;
        r.next++;
        if (r.next < r.nlist) r.pre = ld_copy(r.list + r.next);
    }
}

// Wait (bounded) for every copy still in flight, e.g. before leaving early.
__device__ __forceinline__ void ring_drain(Ring &r)
{
    for (uint32_t i = r.consumed; i < r.issued; i++) {
        mbar_wait_bounded(r.bars + i % (uint32_t)r.stages, (i / (uint32_t)r.stages) & 1u);
    }
    r.consumed = r.issued;
}

// ------------------------------------------------------------------ //
// x staging                                                          //
// ------------------------------------------------------------------ //

// 2^k as a float, for -126 <= k <= 127.
__device__ __forceinline__ float pow2f(int k)
{
    return __uint_as_float((uint32_t)(k + 127) << 23);
}

// hb = silu(gate) * up with the reference's rounding steps,
// src/gguf_forward.c:287-290.
__device__ __forceinline__ float swiglu(float g, float u)
{
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// The signed base-256 digits of four 23-bit integers X_e, given as
// Y_e = X_e + 0x808080 (0 <= Y_e < 2^24): digit k of X_e is byte k of Y_e
// minus 128, so plane k packs byte k of Y_0..Y_3 (a byte transpose), with
// the sign bit of each byte flipped.
__device__ __forceinline__ void digit_planes(const uint32_t *Y, uint32_t &p0, uint32_t &p1, uint32_t &p2)
{
    const uint32_t t0 = __byte_perm(Y[0], Y[1], 0x5140), t1 = __byte_perm(Y[2], Y[3], 0x5140);
    const uint32_t u0 = __byte_perm(Y[0], Y[1], 0x0062), u1 = __byte_perm(Y[2], Y[3], 0x0062);
    p0 = __byte_perm(t0, t1, 0x5410) ^ 0x80808080u;
    p1 = __byte_perm(t0, t1, 0x7632) ^ 0x80808080u;
    p2 = __byte_perm(u0, u1, 0x5410) ^ 0x80808080u;
}

// Stage the phase's input vector in integer form (pk_quant.cuh), for
// PRO_NORM the RMSNorm'ed vector of src/gguf_forward.c:24-40
// (o = w * (ss * x), ss = 1 / sqrtf(mean(x^2) + eps)) and for PRO_EMBED_NORM
// the same of the embedding row (bit-exact decode, src/gguf_model.c:314-359).
// A matvec is linear in its input, so the digits hold w * x and the caller
// multiplies each row's sum by the returned ss (1 for the other prologues):
// the block-wide sum of squares is then reduced beside the digits instead
// of before them. All threads of the CTA.
//
// Four threads own a 32-column group (eight columns each, kept in
// registers from one load to the digits), so there are no per-element
// round trips and only two-step shuffles within the quad. Tagged inputs
// (xin_ll) are polled until they carry `tag`.
__device__ __forceinline__ float stage_x(const Phase &p, const int *step, uint8_t *xq, float *xg, uint32_t tag,
                                         int *err)
{
    constexpr int MAXP = 2;  // groups per quad per pass
    __shared__ float red[32];
    const int pro = p.pro, n = p.cols, ng = 2 * p.nunits;
    const bool normed = pro == PRO_NORM || pro == PRO_EMBED_NORM;
    const float *xin = p.xin, *norm = p.norm;
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int quad = tid >> 2, t = tid & 3, nquads = nt >> 2;
    const uint8_t *erow = nullptr;
    int etype = 0;
    if (pro == PRO_EMBED_NORM) {
        erow = p.embd + (size_t)step[0] * p.embd_rb;
        etype = p.embd_type;
    }
    // the stall test hook polls for a tag that never comes, with a short limit
    const uint32_t wtag = p.stall > 0 ? tag + 1u : tag;
    const long long wlimit = p.stall > 0 ? p.stall : LL_WAIT_LIMIT_CYCLES;
    auto load8 = [&](int c0, float *v) {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = 0.0f;
        if (pro == PRO_EMBED_NORM) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (c0 + e < n) v[e] = decode_col_call(etype, erow, c0 + e);
            }
        } else if (pro == PRO_SWIGLU) {
            // hb = silu(gate) * up, src/gguf_forward.c:287-290
            if (c0 < n) {
                float u[8];
                ll_read8x2(p.xin_ll + c0, p.xin_ll + n + c0, min(8, n - c0), wtag, v, u, err, wlimit);
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = swiglu(v[e], u[e]);
            }
        } else if (p.xin_ll != nullptr) {
            if (c0 < n) ll_read8(p.xin_ll + c0, min(8, n - c0), wtag, v, err, wlimit);
        } else if (c0 + 8 <= n) {
            // x was written by other CTAs (possibly in this launch): read L2
            const float4 a = __ldcg(reinterpret_cast<const float4 *>(xin + c0));
            const float4 b = __ldcg(reinterpret_cast<const float4 *>(xin + c0 + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (c0 + e < n) v[e] = __ldcg(xin + c0 + e);
            }
        }
    };
    float ss = 0.0f;  // this thread's share of the sum of squares (normed)
    for (int base = 0; base < ng; base += MAXP * nquads) {
        float v[MAXP][8], nv[MAXP][8];
        if (normed) {
            // the norm weights do not depend on x: their loads are in flight
            // while the inputs are polled
#pragma unroll
            for (int k = 0; k < MAXP; k++) {
                const int c0 = 32 * (base + quad + k * nquads) + 8 * t;
#pragma unroll
                for (int e = 0; e < 8; e++) nv[k][e] = c0 + e < n ? __ldg(norm + c0 + e) : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < MAXP; k++) {
            const int g = base + quad + k * nquads;
            load8(32 * g + 8 * t, v[k]);  // beyond ng: zeros (c0 >= n)
        }
#pragma unroll
        for (int k = 0; k < MAXP; k++) {
            // The shuffles below name all 32 lanes, so the loop may only be
            // left by whole warps: quads past ng run on zeros, store nothing.
            if (base + 8 * warp + k * nquads >= ng) break;
            const int g = base + quad + k * nquads;
            const bool act = g < ng;
            if (normed) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    ss = fmaf(v[k][e], v[k][e], ss);
                    v[k][e] = __fmul_rn(nv[k][e], v[k][e]);
                }
            }
            float amax = 0.0f, sum = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                amax = fmaxf(amax, fabsf(v[k][e]));
                sum += v[k][e];
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
            // amax = m * 2^E with m in [0.5, 1): E from the exponent bits.
            // Groups below 2^-105 (or subnormal) are stored as zero.
            const int E = (int)((__float_as_uint(amax) >> 23) & 255u) - 126;
            const bool live = E >= -104;
            const float f = live ? pow2f(22 - E) : 0.0f;
            // X = v * f rounded to nearest even (exact: |v * f| < 2^22 and f
            // is a power of two) via the float 1.5 * 2^23 + X, whose bits
            // are 0x4B400000 + X; Y = X + 0x808080 carries X's signed
            // base-256 digits, X = d0 + 2^8 d1 + 2^16 d2, |dk| <= 128
            uint32_t Y[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                Y[e] = __float_as_uint(fmaf(v[k][e], f, 12582912.0f)) - (0x4B400000u - 0x808080u);
            }
            uint32_t w0[2], w1[2], w2[2];
            digit_planes(Y, w0[0], w1[0], w2[0]);
            digit_planes(Y + 4, w0[1], w1[1], w2[1]);
            // digit sums of the thread's eight columns, then per 16-column
            // half: threads (0,1) and (2,3)
            int ds0 = dp4a_ss(w0[1], 0x01010101u, dp4a_ss(w0[0], 0x01010101u, 0));
            int ds1 = dp4a_ss(w1[1], 0x01010101u, dp4a_ss(w1[0], 0x01010101u, 0));
            int ds2 = dp4a_ss(w2[1], 0x01010101u, dp4a_ss(w2[0], 0x01010101u, 0));
            ds0 += __shfl_xor_sync(0xFFFFFFFFu, ds0, 1);
            ds1 += __shfl_xor_sync(0xFFFFFFFFu, ds1, 1);
            ds2 += __shfl_xor_sync(0xFFFFFFFFu, ds2, 1);
            if (!act) continue;
            uint8_t *q = xq + (g >> 1) * XQ_UNIT_BYTES + (g & 1) * 96 + 8 * t;
            *reinterpret_cast<uint2 *>(q) = make_uint2(w0[0], w0[1]);
            *reinterpret_cast<uint2 *>(q + 32) = make_uint2(w1[0], w1[1]);
            *reinterpret_cast<uint2 *>(q + 64) = make_uint2(w2[0], w2[1]);
            float *gi = xg + (g >> 1) * XG_UNIT_WORDS + (g & 1) * 8;
            if (t == 0) {
                gi[0] = live ? pow2f(E - 22) : 0.0f;
                gi[1] = sum;
                gi[2] = __int_as_float(ds0);
                gi[3] = __int_as_float(ds1);
                gi[4] = __int_as_float(ds2);
            } else if (t == 2) {
                gi[5] = __int_as_float(ds0);
                gi[6] = __int_as_float(ds1);
                gi[7] = __int_as_float(ds2);
            }
        }
    }
    if (normed) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;  // read after the barrier below, rewritten next phase
    }
    __syncthreads();
    if (!normed) return 1.0f;
    // RMSNorm scale, src/gguf_forward.c:24-40 (sequential sum there; a
    // block-wide tree here)
    float tot = 0.0f;
    for (int w = 0; w < (nt >> 5); w++) tot += red[w];
    float m = __fdiv_rn(tot, (float)n);
    m = __fadd_rn(m, p.eps);
    return __fdiv_rn(1.0f, __fsqrt_rn(m));
}

// ------------------------------------------------------------------ //
// Tile compute                                                       //
// ------------------------------------------------------------------ //

template <int T>
__device__ __forceinline__ float unit_dot(const uint8_t *row, int u, int nblk, int cols, const XUnit &x,
                                          const uint8_t *xq, const float *xg)
{
    if (T == T_Q4_K) return unit_q4k(row, u, x);
    if (T == T_Q5_K) return unit_q5k(row, u, x);
    if (T == T_Q6_K) return unit_q6k(row, u, x);
    if (T == T_Q4_0) return unit_q4_0(row, u, nblk, x);
    if (T == T_Q8_0) return unit_q8_0(row, u, nblk, x);
    return unit_float(T, row, u, cols, xq, xg);
}

// Row sums of a tile: lane i (< nr) returns row i's dot. Rows go in
// unrolled chunks of RU (independent dp4a chains for ILP, accumulated in
// registers); units are taken 32 at a time, one per lane, and each row is
// reduced over the warp once.
template <int T>
__device__ __forceinline__ float tile_rows(const uint8_t *ra, uint64_t rba, int nr, int nunits, int cols,
                                          const uint8_t *xq, const float *xg, int lane)
{
    constexpr int RU = 4;
    const int nblk = cols / block_weights(T);
    float a = 0.0f;
    for (int i0 = 0; i0 < nr; i0 += RU) {
        float va[RU];
#pragma unroll
        for (int j = 0; j < RU; j++) va[j] = 0.0f;
        for (int u0 = 0; u0 < nunits; u0 += 32) {
            const int u = u0 + lane;
            if (u < nunits) {
                XUnit x;
                if (T != T_F32 && T != T_F16) load_xunit(xq, xg, u, x);
#pragma unroll
                for (int j = 0; j < RU; j++) {
                    if (i0 + j < nr) va[j] += unit_dot<T>(ra + (size_t)(i0 + j) * rba, u, nblk, cols, x, xq, xg);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < RU; j++) {
            const float sa = warp_sum(va[j]);
            if (lane == i0 + j) a = sa;
        }
    }
    return a;
}

// Format sets a kernel is compiled for (bit t = GGML type t): a kernel
// carries only the unit loops of the formats its model uses, which keeps
// its code small enough for the instruction caches.
__host__ __device__ constexpr unsigned tbit(int t)
{
    return 1u << t;
}
constexpr unsigned FMT_ALL =
    tbit(T_F32) | tbit(T_F16) | tbit(T_Q4_0) | tbit(T_Q8_0) | tbit(T_Q4_K) | tbit(T_Q5_K) | tbit(T_Q6_K);

template <unsigned MASK>
__device__ __forceinline__ float tile_dispatch(int type, const uint8_t *ra, uint64_t rba, int nr, int nunits,
                                               int cols, const uint8_t *xq, const float *xg, int lane)
{
#define PK_CASE(T)                                                          \
    case T:                                                                 \
        if constexpr ((MASK & tbit(T)) != 0u) {                             \
            return tile_rows<T>(ra, rba, nr, nunits, cols, xq, xg, lane); \
        }                                                                   \
        break;
    switch (type) {
        PK_CASE(T_Q4_K)
        PK_CASE(T_Q5_K)
        PK_CASE(T_Q6_K)
        PK_CASE(T_Q4_0)
        PK_CASE(T_Q8_0)
        PK_CASE(T_F32)
        PK_CASE(T_F16)
    default: break;
    }
#undef PK_CASE
    return 0.0f;
}

// Compute tile t of phase p from its ring slot and apply the epilogue.
// nscale: stage_x's row-sum multiplier; rope: this position's cos/sin
// pairs (EPI_QKV); tag: the step's tag for
// tagged outputs and the residual. MASK: the formats compiled in.
// Rows in column chunks (p.nchunk > 1): each chunk's sum adds to racc and
// the epilogue runs after the last chunk.
template <unsigned MASK>
__device__ __forceinline__ void run_tile(const Phase &p, int t, int chunk, const uint8_t *buf, const uint8_t *xq,
                                         const float *xg, int token, int pos, const float *rope, uint32_t tag,
                                         int *err, int lane, unsigned long long *cta_amax, float &racc,
                                         float nscale)
{
    const MvSeg &s = find_seg(p, t);
    const int r0 = (t - s.tile0) * s.R;
    const int nr = min(s.R, s.rows - r0);
    uintptr_t st = reinterpret_cast<uintptr_t>(s.w) + (uintptr_t)r0 * s.rb;
    // the residual word is issued before the dot products so its L2 latency
    // overlaps them (it was written phases ago; checked after)
    uint64_t resw = 0;
    if (p.epi == EPI_ADD && p.res_ll != nullptr && lane < nr && (p.nchunk == 1 || chunk == p.nchunk - 1)) {
        resw = ld_ll(p.res_ll + r0 + lane);
    }
    // one call of the unrolled tile loop for both cases: a whole tile, or one
    // column chunk of a row (weights relative to the chunk start, x at the
    // chunk's units)
    int nu = p.nunits, ccols = p.cols, u0 = 0;
    if (p.nchunk > 1) {
        u0 = chunk * p.cunits;
        nu = min(p.cunits, p.nunits - u0);
        ccols = min(64 * nu, p.cols - 64 * u0);
        st += (uintptr_t)chunk * (uintptr_t)p.cbytes;
    }
    float va = tile_dispatch<MASK>(s.type, buf + (st & 15), s.rb, nr, nu, ccols, xq + (size_t)u0 * XQ_UNIT_BYTES,
                                   xg + (size_t)u0 * XG_UNIT_WORDS, lane);
    if (p.nchunk > 1) {
        racc += va;
        if (chunk < p.nchunk - 1) return;
        va = racc;
        racc = 0.0f;
    }
    va *= nscale;  // the RMSNorm scale of a normed input (stage_x), else 1
    // Epilogue: lane i owns row r0 + i.
    const int r = r0 + lane;
    if (p.epi == EPI_QKV) {
        // RoPE pairs (2i, 2i+1) sit in neighbouring lanes (R and r0 are even).
        const float other = __shfl_xor_sync(0xFFFFFFFFu, va, 1);
        if (lane < nr) {
            float v = va;
            const int d = r % p.hs;
            if (s.kind != KIND_V && (d & ~1) < p.rope_dim) {
                // rope_head, src/gguf_forward.c:50-66 (cos/sin from the host table)
                const int i0 = d & ~1;
                const float c = rope[i0], sn = rope[i0 + 1];
                const float v0 = (d & 1) ? other : va, v1 = (d & 1) ? va : other;
                v = (d & 1) ? __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, c))
                            : __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, sn));
            }
            if (s.kind == KIND_Q) {
                st_ll(p.q_ll + r, v, tag);
            } else {
                // the cache row serves later steps; this step reads the tagged copy
                const size_t cache_row = ((size_t)p.layer * p.seq_len + pos) * p.kv_dim;
                void *cache = s.kind == KIND_K ? p.kc : p.vc;
                if (p.kv_half) {
                    kv_store(static_cast<__half *>(cache), cache_row + r, v);
                } else {
                    kv_store(static_cast<float *>(cache), cache_row + r, v);
                }
                st_ll((s.kind == KIND_K ? p.k_ll : p.v_ll) + r, v, tag);
            }
        }
    } else if (p.epi == EPI_LOGITS) {
        // logits + greedy argmax: the warp's best (value, lowest row) goes to
        // the CTA's slot; the CTA's to the global one at the end of the phase
        unsigned long long key = 0ull;
        bool bad = false;
        if (lane < nr) {
            const int gr = p.voc0 + r;  // vocabulary index
            p.y[gr] = va;
            for (int q = 0; q < p.world; q++) {
                if (q != p.rank) reinterpret_cast<float *>(p.peer[q])[gr] = va;
            }
            if (isfinite(va)) {
                key = ((unsigned long long)order_key(va) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)gr);
            } else {
                bad = true;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, key, o);
            key = other > key ? other : key;
        }
        if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) cta_amax[1] = 1ull;
        if (lane == 0 && key != 0ull) atomicMax(cta_amax, key);
    } else if (p.epi == EPI_PEER) {
        // partial row of a split matrix: to the rank that reduces it
        if (lane < nr) {
            int q = 0;
            while (q + 1 < p.world && r >= p.own0[q + 1]) q++;
            st_ll_sys(p.peer[q] + (size_t)p.rank * p.own_max + (r - p.own0[q]), va, tag);
        }
    } else if (lane < nr) {
        float out = va;
        if (s.kind == KIND_UP) {
            // an up row: hb = silu(gate) * up with this row's gate, which a
            // gate tile of the same phase writes to y_ll[r] (another warp;
            // a warp takes its gate tiles before its up tiles)
            out = swiglu(ll_read(p.y_ll + r, tag, err), va);
        }
        if (p.epi == EPI_ADD) {
            // residual stream, src/gguf_forward.c:274-276,297-299 (layer 0's input
            // is the embedding row, decoded again here)
            const float res = p.res_ll == nullptr ? decode_col_call(p.embd_type, p.embd + (size_t)token * p.embd_rb, r)
                              : ll_is(resw, tag)    ? ll_val(resw)
                                                    : ll_read(p.res_ll + r, tag, err);
            out = __fadd_rn(res, va);
        }
        if (p.y_ll != nullptr) {
            st_ll(p.y_ll + s.yoff + r, out, tag);
        } else {
            p.y[s.yoff + r] = out;
        }
    }
}

// ------------------------------------------------------------------ //
// All-reduce over the tensor-parallel ranks                          //
// ------------------------------------------------------------------ //

// Item it of an all-reduce phase on this rank: elements
// [it * blockDim.x, ...) of the slice it reduces. Each element is the sum,
// in rank order, of the ranks' partials (tagged words the ranks' EPI_PEER
// epilogues wrote to this rank's receive buffer xin_ll[q][e]) plus the
// residual, and goes as a tagged word to every rank's output vector.
__device__ __forceinline__ void ar_item(const Phase &p, int it, const int *step, uint32_t tag, int *err)
{
    const int e = it * blockDim.x + threadIdx.x;
    if (e >= p.own[p.rank]) return;
    const int g = p.own0[p.rank] + e;  // element of the full vector
    float sum = ll_read(p.xin_ll + e, tag, err);
    for (int q = 1; q < p.world; q++) sum = __fadd_rn(sum, ll_read(p.xin_ll + (size_t)q * p.own_max + e, tag, err));
    const float res = p.res_ll != nullptr ? ll_read(p.res_ll + g, tag, err)
                                          : decode_col_call(p.embd_type, p.embd + (size_t)step[0] * p.embd_rb, g);
    const float out = __fadd_rn(res, sum);
    for (int q = 0; q < p.world; q++) st_ll_sys(p.peer[q] + g, out, tag);
}

// ------------------------------------------------------------------ //
// Attention                                                          //
// ------------------------------------------------------------------ //

// Positions one attention item covers at least: one pass of a CTA's
// warps (8 warps x 32 lanes, one position per lane). Splitting shorter
// spans over more CTAs was measured slower at ~130 positions (the merge's
// extra round trip costs more than the parallel tiles save).
constexpr int ATT_MIN_SPAN = 256;

// Splits of a head's positions over CTAs at most: enough items to cover
// the grid at long contexts; none below ATT_MIN_SPAN positions.
__host__ __device__ inline int attn_max_splits(int n_heads, int grid, int seq_len)
{
    int s = grid / n_heads;
    if (s < 1) s = 1;
    const int by_len = (seq_len + ATT_MIN_SPAN - 1) / ATT_MIN_SPAN;
    return s < by_len ? s : by_len;
}

// Positions per item at context length n.
__host__ __device__ inline int attn_span(int n, int max_splits)
{
    const int per = (n + max_splits - 1) / max_splits;
    return per < ATT_MIN_SPAN ? ATT_MIN_SPAN : per;
}

// Positions per shared-memory tile: a K or V tile is <= 8 KB, and a power
// of two between 8 and 64 so that 256 threads split it evenly.
__host__ __device__ inline int attn_tile(int hs)
{
    int t = 64;
    while (t > 8 && t * hs > 2048) t >>= 1;
    return t;
}

// Shared-memory floats an item needs: the query, this step's K and V rows,
// two K and two V tiles, the tile's probabilities and reduction slots.
__host__ __device__ inline int attn_scratch_floats(int hs, int nwarps)
{
    const int T = attn_tile(hs);
    return 3 * hs + 4 * T * hs + T + 2 * nwarps;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Item (h, s): query head h over positions [s * span, s * span + span) of
// the n in the cache, src/gguf_forward.c:233-266 with the softmax of
// src/transformer.c:85-109. The head's K/V rows stream through shared
// memory in double-buffered tiles of T positions (16-byte cp.async); per
// tile, tpp = 256 / T threads score each position (q . K[t] * scale), the
// online softmax rescales the running sum and output, and threads
// (dimension, position subset) accumulate p * V[t]. With one split the item
// writes the head's output; otherwise the last split to finish (per-head
// counter) merges the splits' (max, sum, output) in split order. q and this
// position's K/V row are tagged words (the QKV phase of the same step wrote
// them; with a half cache they are rounded to half as the cache holds
// them); earlier positions come from the KV cache (KV: float or __half
// entries, widened to float exactly on the read). All threads of the CTA
// (blockDim.x >= 256, a multiple of 32: threads beyond the first 256 take
// no position when scoring).
template <typename KV>
__device__ __forceinline__ void attn_item_t(const Phase &p, int h, int s, int nsplit, int n, int span, float *sm,
                                            uint32_t tag, int *err)
{
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int hs = p.hs, hs4 = hs >> 2, kvd = p.kv_dim, g = h / p.kv_mul;
    const int T = attn_tile(hs), tpp = 256 / T, nsub = nt / hs;
    const int t0 = s * span, t1 = min(n, t0 + span);
    float *qs = sm;                // hs
    float *kcur = qs + hs;         // hs: K row of this step
    float *vcur = kcur + hs;       // hs: V row of this step
    KV *Kt = reinterpret_cast<KV *>(vcur + hs);         // 2 x T x hs (room for floats)
    KV *Vt = reinterpret_cast<KV *>(vcur + hs + 2 * T * hs);  // 2 x T x hs
    float *pt = vcur + hs + 4 * T * hs;  // T probabilities
    float *red = pt + T;           // 2 x nw
    __shared__ int last_sh;

    const bool has_cur = t1 == n;  // the item covers this step's position
    const size_t lbase = (size_t)p.layer * p.seq_len * kvd + (size_t)g * hs;
    const KV *kc = static_cast<const KV *>(p.kc) + lbase, *vc = static_cast<const KV *>(p.vc) + lbase;
    const int ntile = (t1 - t0 + T - 1) / T;
    constexpr int E16 = 16 / (int)sizeof(KV);  // entries per 16-byte copy
    const int hsc = hs / E16;
    // The cached rows of tile k into buffer buf (16-byte cp.async, one
    // commit group); this step's row, which the cache may not hold yet, is
    // skipped and put in by put_cur.
    auto load_rows = [&](int k, int buf) {
        const int tb = t0 + k * T, tc = min(T, t1 - tb);
        KV *K = Kt + buf * T * hs, *V = Vt + buf * T * hs;
        for (int i = tid; i < tc * hsc; i += nt) {
            const int r = i / hsc, c = (i - r * hsc) * E16;
            if (tb + r != n - 1) {
                cp_async16(K + r * hs + c, kc + (size_t)(tb + r) * kvd + c);
                cp_async16(V + r * hs + c, vc + (size_t)(tb + r) * kvd + c);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto put_cur = [&](int k, int buf) {
        const int r = n - 1 - (t0 + k * T);
        if (!has_cur || r < 0 || r >= T) return;
        KV *K = Kt + buf * T * hs, *V = Vt + buf * T * hs;
        for (int i = tid; i < hs; i += nt) {
            kv_store(K, (size_t)r * hs + i, kcur[i]);
            kv_store(V, (size_t)r * hs + i, vcur[i]);
        }
    };
    // The first two tiles' cached rows do not depend on this step: they are
    // in flight while q and this position's k, v arrive.
    load_rows(0, 0);
    if (ntile > 1) load_rows(1, 1);

    const KV *kc0 = static_cast<const KV *>(p.kc);
    for (int i = tid; i < hs; i += nt) {
        qs[i] = ll_read(p.aq_ll + (size_t)h * hs + i, tag, err);
        if (has_cur) {
            // this step's row as the cache holds it
            kcur[i] = kv_round(kc0, ll_read(p.ak_ll + (size_t)g * hs + i, tag, err));
            vcur[i] = kv_round(kc0, ll_read(p.av_ll + (size_t)g * hs + i, tag, err));
        }
    }
    __syncthreads();
    put_cur(0, 0);
    if (ntile > 1) put_cur(1, 1);

    float m_run = -INFINITY, l_run = 0.0f, o_acc = 0.0f;
    const int pr = tid / tpp, pi = tid - pr * tpp;  // scoring: position pr of the tile (< T: a position), part pi
    const int od = tid % hs, osub = tid / hs;       // output: dimension od, position subset osub
    for (int k = 0; k < ntile; k++) {
        const int buf = k & 1, tb = t0 + k * T, tc = min(T, t1 - tb);
        // tiles k and (if any) k + 1 are in flight: wait for k
        if (k + 1 < ntile) {
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const KV *K = Kt + buf * T * hs, *V = Vt + buf * T * hs;
        // scores: tpp threads per position, float4 slices i, i + tpp, ...
        float acc = 0.0f;
        if (pr < tc) {  // pr >= T for threads beyond the first 256, and tc <= T
            const float4 *q4 = reinterpret_cast<const float4 *>(qs);
            for (int d4 = pi; d4 < hs4; d4 += tpp) {
                const float4 kv = kv_load4(K, (size_t)pr * hs + 4 * d4), qv = q4[d4];
                acc = fmaf(qv.x, kv.x, acc);
                acc = fmaf(qv.y, kv.y, acc);
                acc = fmaf(qv.z, kv.z, acc);
                acc = fmaf(qv.w, kv.w, acc);
            }
        }
        for (int o = tpp >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        const float sc = pr < tc ? acc * p.scale : -INFINITY;
        const float wmax = warp_max(sc);
        if (lane == 0) red[warp] = wmax;
        __syncthreads();
        float mt = red[0];
        for (int w = 1; w < nw; w++) mt = fmaxf(mt, red[w]);
        const float m_new = fmaxf(m_run, mt);
        const float e = pr < tc ? expf(sc - m_new) : 0.0f;
        if (pi == 0 && pr < T) pt[pr] = e;
        const float wsum = warp_sum(pi == 0 ? e : 0.0f);
        if (lane == 0) red[nw + warp] = wsum;
        __syncthreads();
        float lt = 0.0f;
        for (int w = 0; w < nw; w++) lt += red[nw + w];
        const float alpha = expf(m_run - m_new);  // 0 on the first tile (m_run = -inf)
        l_run = fmaf(l_run, alpha, lt);
        m_run = m_new;
        if (osub < nsub) {
            float ov = o_acc * alpha;
            for (int t = osub; t < tc; t += nsub) ov = fmaf(pt[t], kv_load(V, (size_t)t * hs + od), ov);
            o_acc = ov;
        }
        __syncthreads();  // tile buffer, pt and red are reused
        if (k + 2 < ntile) {
            load_rows(k + 2, buf);
            put_cur(k + 2, buf);
        }
    }

    // sum the position subsets (the K tiles are free now)
    float *osum = vcur + hs;
    if (osub < nsub) osum[osub * hs + od] = o_acc;
    __syncthreads();
    const int stride = hs + 2;
    for (int d = tid; d < hs; d += nt) {
        float O = 0.0f;
        for (int j = 0; j < nsub; j++) O += osum[j * hs + d];
        if (nsplit == 1) {
            st_ll(p.aout_ll + (size_t)h * hs + d, O / l_run, tag);
        } else {
            float *P = p.part + ((size_t)h * p.nsplit_max + s) * stride;
            P[2 + d] = O;
            if (d == 0) {
                P[0] = m_run;
                P[1] = l_run;
            }
        }
    }
    if (nsplit == 1) return;

    __threadfence();
    __syncthreads();
    if (tid == 0) last_sh = (atomicAdd(p.count + h, 1u) == (unsigned)(nsplit - 1));
    __syncthreads();
    if (!last_sh) return;
    __threadfence();
    const float *P = p.part + (size_t)h * p.nsplit_max * stride;
    float MM = -INFINITY;
    for (int j = 0; j < nsplit; j++) MM = fmaxf(MM, __ldcg(P + (size_t)j * stride));
    float LL = 0.0f;
    for (int j = 0; j < nsplit; j++) {
        LL = fmaf(__ldcg(P + (size_t)j * stride + 1), expf(__ldcg(P + (size_t)j * stride) - MM), LL);
    }
    for (int d = tid; d < hs; d += nt) {
        float O = 0.0f;
        for (int j = 0; j < nsplit; j++) {
            O = fmaf(__ldcg(P + (size_t)j * stride + 2 + d), expf(__ldcg(P + (size_t)j * stride) - MM), O);
        }
        st_ll(p.aout_ll + (size_t)h * hs + d, O / LL, tag);
    }
    if (tid == 0) p.count[h] = 0;
}

// Attention item over a float or a half KV cache.
__device__ __forceinline__ void attn_item(const Phase &p, int h, int s, int nsplit, int n, int span, float *sm,
                                          uint32_t tag, int *err)
{
    if (p.kv_half) {
        attn_item_t<__half>(p, h, s, nsplit, n, span, sm, tag, err);
    } else {
        attn_item_t<float>(p, h, s, nsplit, n, span, sm, tag, err);
    }
}

}  // namespace pk
