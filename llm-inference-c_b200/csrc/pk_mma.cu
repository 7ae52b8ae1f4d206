// pk_mma.cu - the batched fused dequant-matmul on the sm_100a tensor cores:
// Y[b][r] = sum_k W[r][k] * x_b[k] for up to 64 activation vectors x_b that
// share one pass over the packed Q4_K, Q5_K or Q6_K weights (the matmul
// form of the matvec, src/gguf_model.c:693-771, for several sequences at
// once).
//
// Operands (fp16 products are exact in the fp32 accumulator):
//   A (weights): per super-block of 256 columns, the integers sc_j * q
//       (at most 63 * 15 for Q4_K, 63 * 31 for Q5_K: below 2048, exact in
//       fp16), one LOP3 (two for Q5_K, whose fifth bit comes from qh) and
//       one HFMA2 per two weights, written by the dequantising threads
//       straight into tensor memory (tcgen05.st: row = lane, two fp16 per
//       column); the super-block scales d and dmin stay out of the product
//       and are applied in fp32 when the accumulator is read out. A second
//       operand A2 (shared memory) holds the 6-bit mins m_j, twice.
//   B (activations, shared memory): each 256-column piece of every x_b,
//       scaled by a power of two so that its largest magnitude is below
//       2^10, split into two fp16 parts hi = fp16(x) and lo = fp16(x - hi)
//       (22 significant bits together), at MMA columns 2b and 2b + 1. B2
//       holds the 32-column sums of the scaled piece (the min term
//       sum_j m_j * xsum_j): row b, the hi parts at k 0-7 and the lo parts
//       at k 8-15, so that one MMA adds both.
//   D = A x B (N = 2n rounded up to 16) and D2 = A2 x B2 (N2 = n rounded up
//       to 16) in TMEM, fp32, M = 128 rows, read out once per super-block:
//       y[b] += (d * (D[2b] + D[2b+1]) - dmin * D2[b]) / scale.
//
// One CTA per SM, warp-specialised, every hand-off an mbarrier:
//   warps 0-7   dequantise into A: thread t owns weight row t % 128 of the
//               tile (= TMEM lane); warps 0-3 take the low-nibble sub-block
//               of each 64-column step, warps 4-7 the high-nibble one;
//   warps 8-15  read the accumulators out: thread t owns tile row (= TMEM
//               lane) t % 128, warps 8-11 vectors 0-31, warps 12-15 vectors
//               32-63, and keep the running sums of the tile piece;
//   warp 16     loads the weight super-blocks of the tile (128 rows x 144
//               bytes, one 2D TMA tensor copy each, plus the 64 scales of
//               that x piece) into a 4-deep ring;
//   warp 17     bulk-copies the staged x of each 64-column step into a ring
//               as deep as shared memory allows (7 steps at n = 64, 32 at
//               n <= 8);
//   warp 18     allocates TMEM and issues the MMAs from one lane, committing
//               to the barriers that free the A and B slots and publish the
//               accumulators; two accumulator sets let the readout of one
//               super-block overlap the MMAs of the next.
// Dequantisation and readout run on separate warps so that neither waits
// for the other: the A ring keeps filling while a super-block is read out.
// Work units are (row tile, super-block) pairs, split evenly over the CTAs
// in row-tile-major order. A tile split over several CTAs leaves one partial
// sum per CTA; for each block of 32 rows x 32 vectors the last CTA to
// finish it adds the partials up in CTA order (a fixed order: the result
// does not depend on timing). Two launches per call: the x staging kernel,
// then this one.
//
// Shared-memory operands (B, B2, A2) are fp16, K-major, without swizzle:
// core matrices of 8 rows x 16 bytes, rows 16 bytes apart. A step tile of
// 64 columns is [8 column chunks][rows][16 bytes]; element (row, k) sits at
//     (k / 8) * chunk_bytes + row * 16 + pos(k % 8) * 2,
// chunk_bytes = N * 16 (the descriptors' leading offset; their stride offset
// is 128 bytes, the next 8 rows). pos() permutes each run of 8 columns as
// {0, 2, 1, 3, 4, 6, 5, 7}: the order in which one LOP3 takes the nibbles
// out of a 32-bit word of packed weights. A in tensor memory holds the same
// 16-byte runs, in the same order, in four consecutive columns (the sum over
// k does not depend on the order as long as A and B agree).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/gguf_cuda.h"
#include "pk_mma.h"
#include "pk_quant.cuh"
#include "pk_stream.cuh"

namespace pk {
namespace mm {

constexpr int TM = 128;    // weight rows per tile (MMA M)
constexpr int NMAX = 128;  // MMA N at most: 2 parts x 64 vectors
constexpr int VMAX = 64;   // activation vectors per call
constexpr int QK = 256;    // columns per super-block
constexpr int DQ_WARPS = 8, DQ_THREADS = 256;  // warps 0-7 dequantise: two per row group of 32
constexpr int RO_WARP0 = 8, RO_THREADS = 256;   // warps 8-15 read the accumulators out
constexpr int W_PRODUCER = 16, B_PRODUCER = 17, ISSUER = 18;
constexpr int THREADS = 608;
constexpr int SA_MAX = 8, SW_MAX = 4, SB_MAX = 32;  // ring depths at most: A steps, weight super-blocks, x steps
constexpr int SA2 = 3, SINV = 4;  // A2 slots; inverse-scale and row-scale slots (see the readout)
constexpr int A2_BYTES = TM * 32;  // [2 chunks][128 rows][16 B]
// Barriers
enum {
    FULL_A = 0,
    EMPTY_A = FULL_A + SA_MAX,
    FULL_W = EMPTY_A + SA_MAX,
    EMPTY_W = FULL_W + SW_MAX,
    ACC_FULL = EMPTY_W + SW_MAX,
    ACC_EMPTY = ACC_FULL + 2,
    DRAIN = ACC_EMPTY + 2,
    FULL_B = DRAIN + 1,
    EMPTY_B = FULL_B + SB_MAX,
    NBARS = EMPTY_B + SB_MAX
};
// Shared-memory layout (offsets from a 128-byte aligned base). The A
// operand lives in tensor memory, so shared memory holds the weight ring,
// the x ring and the small per-super-block tables.
constexpr int OFF_BAR = 0;
constexpr int OFF_INV = 1024;  // SINV x 64 inverse scales of the x pieces (readout)
constexpr int OFF_DD = 2048;   // SINV x 128 rows: (d, dmin) of each row's super-block as two fp16 (readout)
constexpr int OFF_A2 = 4096;   // SA2 A2 slots (the mins; Q4_K and Q5_K)
constexpr int B_SLOT_MAX = NMAX * 128 + VMAX * 32;
static_assert(NBARS * 8 <= OFF_INV && OFF_INV + SINV * VMAX * 4 <= OFF_DD && OFF_DD + SINV * TM * 4 <= OFF_A2,
              "barriers, scales");

// Tensor memory (512 columns of 128 lanes x 32 bits):
//   D set s (s = 0, 1):   columns 128 s .. 128 s + 127, fp32, MMA N <= 128
//   D2 set s (Q4_K/Q5_K): columns 256 + 64 s .., one column per vector
//   A ring:               32 columns per 64-k step (row = lane, two fp16 per
//                         column in k order), from column ACOL
constexpr int TMEM_COLS = 512;
constexpr int D2_COL = 256;

// The super-block format: bytes, where its nibbles (qs) and fifth bits (qh)
// start, the depth of the weight ring that shared memory leaves room for,
// and the A ring in tensor memory (src/gguf_quant.c:107-161 Q4_K, :307-345
// Q5_K).
template <int T>
struct Fmt;
// SBB: shared-memory bytes per row and super-block; STEPS: MMA steps of 64
// k per super-block; OFFW: the weight ring's offset; SA, ACOL: A ring slots
// and first column.
template <>
struct Fmt<T_Q4_K> {
    static constexpr int SBB = 144, QS = 16, QH = 0, SW = 4, STEPS = 4, OFFW = OFF_A2 + SA2 * A2_BYTES;
    static constexpr int SA = 4, ACOL = 384;
};
template <>
struct Fmt<T_Q5_K> {
    static constexpr int SBB = 176, QS = 48, QH = 16, SW = 4, STEPS = 4, OFFW = OFF_A2 + SA2 * A2_BYTES;
    static constexpr int SA = 4, ACOL = 384;
};
// Q6_K (src/gguf_quant.c:185-252): 210-byte super-blocks, which no tensor
// map can address (neither the blocks nor, in general, the rows start on 16
// bytes), so each row's block arrives by its own bulk copy of the 224-byte
// aligned window that holds it. Its signed 8-bit scales do not give exact
// fp16 products with q - 32, so each 64-k step holds 32 columns twice: k
// 0-31 as 16 a (q - 32), k 32-63 as b (q - 32) with sc = 16 a + b,
// a in [-8, 7], b in [0, 15] (both exact in fp16), against x staged twice;
// the sum over the step is sum sc (q - 32) x. No mins: no A2, no D2.
template <>
struct Fmt<T_Q6_K> {
    static constexpr int SBB = 224, BLK = 210, SW = 4, STEPS = 8, OFFW = OFF_A2;
    static constexpr int SA = 8, ACOL = 256;
};
template <int T>
struct Lay {
    static constexpr int SBB = Fmt<T>::SBB, SW = Fmt<T>::SW;
    static constexpr int W_TILE = TM * SBB;            // 128 rows x one super-block
    static constexpr int W_BYTES = W_TILE + VMAX * 4;  // + the inverse scales of the x piece
    static constexpr int OFF_W = Fmt<T>::OFFW;
    static constexpr int OFF_B = OFF_W + SW * W_BYTES;
    static_assert(OFF_W % 128 == 0 && W_BYTES % 128 == 0, "TMA destinations");
    static_assert(OFF_B + 3 * B_SLOT_MAX + 128 <= 227 * 1024 - 1024, "at least 3 x steps of N = 128");
    static_assert(SW <= SW_MAX && Fmt<T>::SA <= SA_MAX, "ring barriers");
    static_assert(Fmt<T>::ACOL + 32 * Fmt<T>::SA <= TMEM_COLS, "A ring inside tensor memory");
    // a readout slot (SINV deep) is rewritten at the start of super-block
    // j + SINV; the dequantisers then have waited for the MMAs of a step of
    // super-block j + 2 or later (see the readout) only if SA < 2 STEPS
    static_assert(Fmt<T>::SA < 2 * Fmt<T>::STEPS && SINV >= 4, "readout slot lifetimes");
};

// Position of column k (mod 8) inside its 16-byte run: 1 <-> 2, 5 <-> 6.
__host__ __device__ constexpr int perm8(int i)
{
    return (i == 1 || i == 2 || i == 5 || i == 6) ? (i ^ 3) : i;
}

// CTA owning work unit u when U units are split over G CTAs as
// [c * U / G, (c + 1) * U / G).
__host__ __device__ inline int unit_owner(long long u, long long U, long long G)
{
    return (int)(((u + 1) * G - 1) / U);
}

// UMMA shared-memory descriptor: K-major, no swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor of kind::f16: fp16 A and B, both K-major, fp32 D.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n)
{
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// The same with A in tensor memory: 128 lanes (rows) x 8 columns (16 fp16
// in k order) from column address a_tmem.
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t accum)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}

// Arrive on bar once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 2D TMA tensor copy of the box at (x, y) (x in elements of the innermost
// dimension) into shared memory, completing on bar.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane at taddr and 8 at
// taddr2 (warp w reads lanes 32 (w % 4) .. + 31; an address carries the lane
// in bits 16-31): both loads and their wait in one statement, so that no use
// of the values can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld16x8(uint32_t taddr, uint32_t taddr2, float *v, float *v2)
{
    uint32_t r[24];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%24];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%25];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23])
        : "r"(taddr), "r"(taddr2)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
#pragma unroll
    for (int i = 0; i < 8; i++) v2[i] = __uint_as_float(r[16 + i]);
}

// 16 consecutive fp32 columns at taddr, loaded and waited for in one statement.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v)
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Store 16 32-bit words to consecutive columns of this thread's TMEM lane,
// then wait until the stores are done (the tensor core reads them next).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n\t"
        "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Two quants of w (bits 0-3 and 16-19; Q5_K: 0-4 and 16-20) as the fp16
// pair (sc * q0, sc * q1): 1024 + q by the exponent trick, then
// (1024 + q) * sc - 1024 * sc in one fma, exact because the result is an
// integer below 2048.
template <int FT>
__device__ __forceinline__ uint32_t nib2(uint32_t w, __half2 sc2, __half2 nsc2)
{
    const uint32_t h = (w & (FT == T_Q5_K ? 0x001F001Fu : 0x000F000Fu)) | 0x64006400u;
    const __half2 r = __hfma2(*reinterpret_cast<const __half2 *>(&h), sc2, nsc2);
    return *reinterpret_cast<const uint32_t *>(&r);
}

// Two 6-bit quants of w (bits 0-5 and 16-21) as the fp16 pair
// ((q0 - 32) s, (q1 - 32) s): 1024 + q by the exponent trick, minus 1056,
// times s; each step exact (the products are integers of at most 12 bits).
__device__ __forceinline__ uint32_t q6pair(uint32_t w, __half2 s2)
{
    const uint32_t h = (w & 0x003F003Fu) | 0x64006400u;
    const __half2 r = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&h), __float2half2_rn(1056.0f)), s2);
    return *reinterpret_cast<const uint32_t *>(&r);
}

// mbarrier.try_wait with a suspend-time hint: the thread sleeps until the
// phase completes (or about a millisecond passes) instead of spinning, so
// waiting warps take no issue slots from the working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// One lane of a converged warp (the same lane every time).
__device__ __forceinline__ bool elect_one()
{
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// The slow path of wait_or_abort, out of line: the kernel's code stays
// small enough for the instruction caches that its eleven warps share.
__device__ __noinline__ bool wait_or_abort_slow(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
            *abort_flag = 1;
            atomicOr(err, ERR_TIMEOUT_MV);
            return false;
        }
    }
    return true;
}

// Bounded wait that also gives up once another thread has aborted the CTA;
// a thread that runs out of time records the timeout and aborts the CTA.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    return mbar_try_wait_sleep(bar, parity) || wait_or_abort_slow(bar, parity, abort_flag, err);
}

// wait_or_abort with one answer for the whole warp (every lane calls it), so
// that the warp's later collective instructions stay converged.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    const bool got = wait_or_abort(bar, parity, abort_flag, err);
    return __all_sync(0xFFFFFFFFu, got);
}

constexpr int MSEG = 3;  // weight matrices (segments) of one launch, all with the same columns

// The weight matrices of one launch as 2D tensors of bytes [rows][row
// bytes], box [128 rows][one super-block's bytes] (one row tile).
struct MmMaps {
    CUtensorMap m[MSEG];
};

struct MmArgs {
    int nseg;               // segments: row tiles [tile0[s], tile0[s + 1]) are matrix s
    int tile0[MSEG + 1];
    int seg_rows[MSEG];
    float *seg_y[MSEG];     // [n][rows of the segment]
    const uint8_t *seg_w[MSEG];  // Q6_K: row 0 of each matrix, and its row bytes
    uint64_t seg_rb[MSEG];
    int nsb;                // super-blocks per row
    const uint8_t *xs;      // staged x: [nsb][STEPS][8 chunks][N rows][16 B]
    const uint8_t *x2s;     // staged x sums: [nsb][2 chunks (hi, lo)][N2 rows][16 B]
    const float *xinv;      // [nsb][64] inverse scales of the staged pieces
    int n, N, N2;           // vectors, MMA N of D (hi and lo column per vector) and of D2 (one per vector)
    int sb, b_slot;         // x ring depth and slot bytes
    int U;                  // work units (row tiles x super-blocks)
    int G;                  // CTAs
    int maxp;               // partial slots per tile
    float *ypart;           // [tiles][maxp][n][128]
    unsigned int *arrived;  // [tiles][8 warps] CTAs done with that block (reset by the last)
    int *err;
};

// Store the sums of one tile piece: acc[b] = vector b0 + b of tile row
// row. A tile owned by one CTA goes straight to y. Otherwise the piece goes
// to the CTA's partial slot; per read-out warp (32 rows x 32 vectors) a
// counter of the CTAs done with that block names the last one, which adds
// the pieces in CTA order (no barrier between warps: an aborted warp blocks
// none).
// Out of line and rare (once per tile piece): it keeps the kernel small.
// T: the tile's index over all segments (partial slots, owners); lt: its
// index inside its matrix, whose rows and output are rows / y.
__device__ __noinline__ void flush_piece(const float *acc, float *y, float *ypart, unsigned int *arrived, int rows,
                                         int n, int nsb, int U, int G, int maxp, int T, int lt, int c, int row,
                                         int b0)
{
    const int warp = (threadIdx.x >> 5) - RO_WARP0, lane = threadIdx.x & 31;
    const int r = lt * TM + row;
    const int c0 = unit_owner((long long)T * nsb, U, G), c1 = unit_owner((long long)T * nsb + nsb - 1, U, G);
    const int nb = min(32, n - b0);
    if (c0 == c1) {
        if (r < rows)
            for (int b = 0; b < nb; b++) y[(size_t)(b0 + b) * rows + r] = acc[b];
        return;
    }
    float *yp = ypart + (size_t)T * maxp * n * TM;
    for (int b = 0; b < nb; b++) yp[((size_t)(c - c0) * n + b0 + b) * TM + row] = acc[b];
    __threadfence();
    __syncwarp();
    unsigned int last = 0;
    if (lane == 0) {
        const unsigned int seen = atomicAdd(arrived + (size_t)T * DQ_WARPS + warp, 1u);
        last = seen == (unsigned int)(c1 - c0);
        if (last) arrived[(size_t)T * DQ_WARPS + warp] = 0u;  // ready for the next call
    }
    last = __shfl_sync(0xFFFFFFFFu, last, 0);
    if (last) {
        __threadfence();
        if (r < rows) {
            // piece by piece, the 32 vectors' loads of a piece in flight together
            float sum[32];
#pragma unroll
            for (int b = 0; b < 32; b++) sum[b] = 0.0f;
            for (int k = 0; k <= c1 - c0; k++) {
                const float *pk = yp + ((size_t)k * n + b0) * TM + row;
#pragma unroll
                for (int b = 0; b < 32; b++)
                    if (b < nb) sum[b] += __ldcg(pk + (size_t)b * TM);
            }
#pragma unroll
            for (int b = 0; b < 32; b++)
                if (b < nb) y[(size_t)(b0 + b) * rows + r] = sum[b];
        }
    }
}

__device__ __forceinline__ int seg_of(const MmArgs &a, int T)
{
    int sg = 0;
    while (sg + 1 < a.nseg && T >= a.tile0[sg + 1]) sg++;
    return sg;
}

template <int FT>
__global__ void __launch_bounds__(THREADS, 1) qk_mm_kernel(const __grid_constant__ MmMaps maps, MmArgs a)
{
    constexpr int SBB = Fmt<FT>::SBB, SW = Fmt<FT>::SW, STEPS = Fmt<FT>::STEPS;
    constexpr int W_TILE = Lay<FT>::W_TILE, W_BYTES = Lay<FT>::W_BYTES, OFF_B = Lay<FT>::OFF_B;
    constexpr int OFF_W = Lay<FT>::OFF_W, SA = Fmt<FT>::SA, ACOL = Fmt<FT>::ACOL;
    constexpr bool Q6 = FT == T_Q6_K;
    extern __shared__ __align__(128) uint8_t sm_raw[];
    uint8_t *sm = sm_raw + ((128u - (smem_u32(sm_raw) & 127u)) & 127u);
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    float *inv_s = reinterpret_cast<float *>(sm + OFF_INV);
    const int c = blockIdx.x;
    // this CTA's units [u0, u0 + nu): tile T0, super-block s0 first
    const int u0 = (int)((long long)c * a.U / a.G);
    const int nu = (int)((long long)(c + 1) * a.U / a.G) - u0;
    const int T0 = u0 / a.nsb, s0 = u0 - T0 * a.nsb;
    const int N = a.N, SB = a.sb;

    if (warp == ISSUER) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < SA; i++) {
            mbar_init(bars + FULL_A + i, DQ_THREADS);
            mbar_init(bars + EMPTY_A + i, 1);
        }
        for (int i = 0; i < SW; i++) {
            mbar_init(bars + FULL_W + i, 1);
            mbar_init(bars + EMPTY_W + i, DQ_THREADS);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bars + ACC_FULL + i, 1);
            mbar_init(bars + ACC_EMPTY + i, RO_THREADS);
        }
        mbar_init(bars + DRAIN, 1);
        for (int i = 0; i < SB; i++) {
            mbar_init(bars + FULL_B + i, 1);
            mbar_init(bars + EMPTY_B + i, 1);
        }
        fence_mbar_init();
        abort_flag = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t sbase = smem_u32(sm);
    volatile int *abrt = &abort_flag;

    if (warp == W_PRODUCER) {
        // weight super-blocks: one tensor copy of 128 rows x SBB bytes each
        // (rows past the end of the matrix arrive as zeros), then the 64
        // inverse scales of the matching x piece
        const bool leader = elect_one();
        if (leader && !Q6) {
            for (int sg = 0; sg < a.nseg; sg++)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.m[sg])) : "memory");
        }
        const int lane = tid & 31;
        int issued = 0, T = T0, s = s0;
        for (int j = 0; j < nu; j++) {
            const int slot = j % SW;
            if (j >= SW && !warp_wait(bars + EMPTY_W + slot, ((j / SW) - 1) & 1, abrt, a.err)) break;
            uint8_t *dst = sm + OFF_W + slot * W_BYTES;
            const int sg = seg_of(a, T);
            if (Q6) {
                // each row's block in its 16-byte aligned 224-byte window; rows
                // past the matrix are not copied (their sums are never stored)
                const int r0 = (T - a.tile0[sg]) * TM, nr = min(TM, a.seg_rows[sg] - r0);
                if (leader) mbar_expect_tx(bars + FULL_W + slot, (uint32_t)(nr * SBB + VMAX * 4));
                __syncwarp();
                for (int r = lane; r < nr; r += 32) {
                    const uintptr_t src = reinterpret_cast<uintptr_t>(a.seg_w[sg]) +
                                          (uintptr_t)(r0 + r) * a.seg_rb[sg] + (uintptr_t)s * Fmt<T_Q6_K>::BLK;
                    bulk_g2s(dst + r * SBB, reinterpret_cast<const void *>(src & ~(uintptr_t)15), SBB,
                             bars + FULL_W + slot);
                }
                if (leader) bulk_g2s(dst + W_TILE, a.xinv + (size_t)s * VMAX, VMAX * 4, bars + FULL_W + slot);
            } else if (leader) {
                mbar_expect_tx(bars + FULL_W + slot, (uint32_t)W_BYTES);
                tma_load_2d(dst, &maps.m[sg], s * SBB, (T - a.tile0[sg]) * TM, bars + FULL_W + slot);
                bulk_g2s(dst + W_TILE, a.xinv + (size_t)s * VMAX, VMAX * 4, bars + FULL_W + slot);
            }
            __syncwarp();
            issued = j + 1;
            if (++s == a.nsb) {
                s = 0;
                T++;
            }
        }
        // no copy may still be in flight when the CTA exits
        for (int j = max(0, issued - SW); j < issued; j++) mbar_wait_bounded(bars + FULL_W + j % SW, (j / SW) & 1);
    } else if (warp == B_PRODUCER) {
        // one lane copies the staged x of every step into the ring
        if (elect_one()) {
            const uint32_t step_bytes = (uint32_t)N * 128, sum_bytes = (uint32_t)a.N2 * 32;
            int issued = 0, slot = 0, s = s0;
            uint32_t phase = 0;  // parity of the slot's next EMPTY_B completion
            for (int i = 0; i < STEPS * nu; i++) {
                if (i >= SB && !wait_or_abort(bars + EMPTY_B + slot, phase, abrt, a.err)) break;
                const int t = i % STEPS;
                const bool sums = !Q6 && t == STEPS - 1;  // the min term's x sums (Q4_K, Q5_K)
                uint8_t *dst = sm + OFF_B + slot * a.b_slot;
                mbar_expect_tx(bars + FULL_B + slot, step_bytes + (sums ? sum_bytes : 0u));
                bulk_g2s(dst, a.xs + ((size_t)s * STEPS + t) * step_bytes, step_bytes, bars + FULL_B + slot);
                if (sums) bulk_g2s(dst + step_bytes, a.x2s + (size_t)s * sum_bytes, sum_bytes, bars + FULL_B + slot);
                issued = i + 1;
                if (t == STEPS - 1 && ++s == a.nsb) s = 0;
                if (++slot == SB) {
                    slot = 0;
                    if (i >= SB) phase ^= 1u;
                }
            }
            for (int i = max(0, issued - SB); i < issued; i++) mbar_wait_bounded(bars + FULL_B + i % SB, (i / SB) & 1);
        }
        __syncwarp();
    } else if (warp == ISSUER) {
        // One lane issues: the loop between two MMA steps is a short chain
        // of single-thread instructions (the tensor core takes an M = 128,
        // N = 128, K = 16 MMA every 64 cycles; descriptor arithmetic between
        // issues would leave it idle).
        if (elect_one()) {
            const uint32_t idesc = idesc_f16(TM, N), idesc2 = idesc_f16(TM, a.N2);
            // descriptors of slot 0 / chunk pair 0; later ones add (offset >> 4).
            // A of step slot as: tensor-memory columns ACOL + 32 as + 8 kk.
            const uint64_t b_desc0 = sdesc(sbase + OFF_B, N * 16, 128);
            const uint64_t b2_desc0 = sdesc(sbase + OFF_B + N * 128, a.N2 * 16, 128);
            const uint64_t a2_desc0 = sdesc(sbase + OFF_A2, TM * 16, 128);
            const uint32_t b_kstep = (uint32_t)(2 * N * 16) >> 4, b_slot16 = (uint32_t)a.b_slot >> 4;
            const uint32_t a_col0 = tmem + (uint32_t)ACOL;
            bool ok = true;
            int issued = 0, as = 0, bs = 0;
            uint32_t a_ph = 0, b_ph = 0;  // parity of the slots' next FULL completion
            for (int j = 0; j < nu && ok; j++) {
                const int acc = j & 1;
                const uint32_t d_col = tmem + (uint32_t)(acc * 128);
                if (j >= 2 && !wait_or_abort(bars + ACC_EMPTY + acc, ((j / 2) - 1) & 1, abrt, a.err)) break;
                tc_fence_after();
#pragma unroll 1
                for (int t = 0; t < STEPS; t++) {
                    if (!wait_or_abort(bars + FULL_A + as, a_ph, abrt, a.err) ||
                        !wait_or_abort(bars + FULL_B + bs, b_ph, abrt, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ta = a_col0 + (uint32_t)(32 * as);
                    const uint64_t bd = b_desc0 + (uint64_t)(bs * b_slot16);
                    mma_f16_ta(d_col, ta, bd, idesc, t != 0 ? 1u : 0u);
                    mma_f16_ta(d_col, ta + 8, bd + b_kstep, idesc, 1u);
                    mma_f16_ta(d_col, ta + 16, bd + 2 * b_kstep, idesc, 1u);
                    mma_f16_ta(d_col, ta + 24, bd + 3 * b_kstep, idesc, 1u);
                    if (!Q6 && t == STEPS - 1) {
                        // the min term: D2[b] = sum_j m_j (hi_j + lo_j) of the x piece's
                        // 32-column sums (k 0-7 against the hi parts, 8-15 the lo parts)
                        mma_f16(tmem + (uint32_t)(D2_COL + 64 * acc),
                                a2_desc0 + (uint64_t)((j % SA2) * (A2_BYTES >> 4)),
                                b2_desc0 + (uint64_t)(bs * b_slot16), idesc2, 0u);
                    }
                    mma_commit(bars + EMPTY_A + as);
                    mma_commit(bars + EMPTY_B + bs);
                    issued++;
                    if (++as == SA) {
                        as = 0;
                        a_ph ^= 1u;
                    }
                    if (++bs == SB) {
                        bs = 0;
                        b_ph ^= 1u;
                    }
                }
                if (ok) mma_commit(bars + ACC_FULL + acc);
            }
            // MMAs still running after an abort finish before TMEM is freed
            if (issued > 0) {
                mma_commit(bars + DRAIN);
                mbar_wait_bounded(bars + DRAIN, 0);
            }
        }
        __syncwarp();
    } else if (warp >= RO_WARP0) {
        // warps 8-15: read the accumulators out. Thread rt owns tile row
        // row = rt % 128 (TMEM lane row) and the vectors 32 half .. 32 half
        // + 31, half = rt / 128. Per super-block jp (after its MMAs):
        //   acc[b] += inv[b] * (d * (D[2b] + D[2b+1]) - dmin * D2[b])
        // with the row's d, dmin and the x piece's inverse scales from slot
        // jp % SINV. Slot lifetimes: the dequantisers write slot jp % SINV
        // at the start of super-block jp and again at the start of jp +
        // SINV, after the last step of jp + SINV - 1, for which they waited
        // until the MMAs of the step SA before it completed: a step of
        // super-block jp + 2 or later (SA < 2 STEPS, SINV >= 4), whose MMAs
        // the issuer starts only after this readout has freed its
        // accumulator set (ACC_EMPTY, arrived after the last read of the
        // slot).
        const int rt = tid - RO_WARP0 * 32;
        const int row = rt & (TM - 1), half = rt >> 7;
        const int b0 = 32 * half;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t *dd = reinterpret_cast<const uint32_t *>(sm + OFF_DD);
        float acc[32];
#pragma unroll
        for (int b = 0; b < 32; b++) acc[b] = 0.0f;
        int rT = T0, rs = s0;  // tile and super-block of the next readout
        for (int jp = 0; jp < nu; jp++) {
            const int accs = jp & 1;
            if (!warp_wait(bars + ACC_FULL + accs, (jp / 2) & 1, abrt, a.err)) break;
            tc_fence_after();
            const uint32_t hd = dd[(jp % SINV) * TM + row];
            const float d = hf(hd & 0xFFFFu), dmin = hf(hd >> 16);
            const float *iv = inv_s + (jp % SINV) * VMAX + b0;
            const uint32_t col = lane_base + (uint32_t)(accs * 128 + 2 * b0);
            const uint32_t col2 = lane_base + (uint32_t)(D2_COL + 64 * accs + b0);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                if (2 * b0 + 16 * q < N) {
                    float v[16], v2[8];
                    if (Q6) {
                        tmem_ld16(col + 16 * q, v);
                    } else {
                        tmem_ld16x8(col + 16 * q, col2 + 8 * q, v, v2);
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int b = 8 * q + i;
                        const float t1 = d * (v[2 * i] + v[2 * i + 1]);
                        acc[b] = Q6 ? fmaf(iv[b], t1, acc[b]) : fmaf(iv[b], fmaf(-dmin, v2[i], t1), acc[b]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(bars + ACC_EMPTY + accs);
            const bool piece_end = jp == nu - 1 || rs == a.nsb - 1;
            if (piece_end && b0 < a.n) {
                float out[32];
#pragma unroll
                for (int b = 0; b < 32; b++) out[b] = acc[b];
                const int sg = seg_of(a, rT);
                flush_piece(out, a.seg_y[sg], a.ypart, a.arrived, a.seg_rows[sg], a.n, a.nsb, a.U, a.G, a.maxp, rT,
                            rT - a.tile0[sg], c, row, b0);
            }
        if (++rs == a.nsb) {
                rs = 0;
                rT++;
            }
            if (piece_end) {
#pragma unroll
                for (int b = 0; b < 32; b++) acc[b] = 0.0f;
            }
        }
    } else {
        // warps 0-7: dequantise into A. Thread tid owns tile row
        // row = tid % 128; half = tid / 128 picks the sub-block of each step
        // (low or high nibbles). At the start of super-block j the row's
        // (d, dmin) and the x piece's inverse scales go to slot j % SINV for
        // the readout.
        const int row = tid & (TM - 1), half = tid >> 7;
        uint32_t *dd = reinterpret_cast<uint32_t *>(sm + OFF_DD);
        // this warp's TMEM lanes (32 (warp % 4) ..) at the A ring's first column
        const uint32_t a_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)ACOL;
        bool ok = true;
        int as = 0;
        uint32_t ea_ph = 0;  // parity of the A slot's next EMPTY completion
        int dT = T0, ds = s0;  // tile and super-block being dequantised
        for (int j = 0; j < nu && ok; j++) {
            const int ws = j % SW;
            if (!warp_wait(bars + FULL_W + ws, (j / SW) & 1, abrt, a.err)) {
                ok = false;
                break;
            }
            const uint8_t *wslot = sm + OFF_W + ws * W_BYTES;
            if (tid < VMAX) inv_s[(j % SINV) * VMAX + tid] = reinterpret_cast<const float *>(wslot + W_TILE)[tid];
            if constexpr (Q6) {
                // this row's block sits in its window at the block's offset
                // from a 16-byte boundary (an even number: rows and blocks
                // have even sizes)
                const int sg = seg_of(a, dT);
                const uintptr_t gaddr = reinterpret_cast<uintptr_t>(a.seg_w[sg]) +
                                        (uintptr_t)((dT - a.tile0[sg]) * TM + row) * a.seg_rb[sg] +
                                        (uintptr_t)ds * Fmt<T_Q6_K>::BLK;
                const uint8_t *blk = wslot + row * SBB + (gaddr & 15u);
                uint32_t ql[16], qh6[8], scw[2];
                if (half == 0) dd[(j % SINV) * TM + row] = ld_u16(blk + 208);  // d; no mins
                // the two halves of the block (h: columns 128h ..) in a runtime
                // loop, the four steps of a half unrolled: every array index
                // below is a constant, so the words stay in registers
#pragma unroll 1
                for (int h = 0; h < 2 && ok; h++) {
                    ld_words_a2<16>(blk + 64 * h, ql);        // ql bytes 64h .. 64h + 63
                    ld_words_a2<8>(blk + 128 + 32 * h, qh6);  // qh bytes 32h .. 32h + 31
                    ld_words_a2<2>(blk + 192 + 8 * h, scw);   // the signed scales 8h .. 8h + 7
                    if (h == 1) mbar_arrive(bars + EMPTY_W + ws);  // the slot's last read
#pragma unroll
                    for (int m = 0; m < 4; m++) {
                        const int i = STEPS * j + 4 * h + m;
                        if (i >= SA && !warp_wait(bars + EMPTY_A + as, ea_ph, abrt, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();  // the MMAs that read this A slot have completed
                        // step 4h + m: columns 128h + 32m + l of the block
                        const int nsh = m >= 2 ? 4 : 0, hsh = 2 * m, wb = 8 * (m & 1);
                        uint32_t aw[16];  // this half of the step: tensor-memory columns 16 half .. + 15
#pragma unroll
                        for (int cc = 0; cc < 4; cc++) {
                            // columns l = 8cc .. 8cc + 7; scale 8h + 2m + l / 16; this
                            // half's part of sc = 16 a + b: 16 a (k 0-31) or b (k 32-63)
                            const int g = 2 * m + (cc >> 1);
                            const int sc = (int)(int8_t)((scw[g >> 2] >> (8 * (g & 3))) & 255u);
                            const __half2 s2 =
                                __float2half2_rn(half == 0 ? (float)(16 * (sc >> 4)) : (float)(sc & 15));
                            const uint32_t q0 = ((ql[wb + 2 * cc] >> nsh) & 0x0F0F0F0Fu) |
                                                (((qh6[2 * cc] >> hsh) & 0x03030303u) << 4);
                            const uint32_t q1 = ((ql[wb + 2 * cc + 1] >> nsh) & 0x0F0F0F0Fu) |
                                                (((qh6[2 * cc + 1] >> hsh) & 0x03030303u) << 4);
                            aw[4 * cc] = q6pair(q0, s2);
                            aw[4 * cc + 1] = q6pair(q0 >> 8, s2);
                            aw[4 * cc + 2] = q6pair(q1, s2);
                            aw[4 * cc + 3] = q6pair(q1 >> 8, s2);
                        }
                        tmem_st16(a_lane + (uint32_t)(32 * as + 16 * half), aw);
                        tc_fence_before();
                        mbar_arrive(bars + FULL_A + as);
                        if (++as == SA) {
                            as = 0;
                            if (i >= SA) ea_ph ^= 1u;
                        }
                    }
                }
            } else {
                const uint8_t *wrow = wslot + row * SBB;
                const uint4 hdr = *reinterpret_cast<const uint4 *>(wrow);
                uint32_t qh[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // Q5_K: the fifth bits of the 32 byte positions
                if (FT == T_Q5_K) {
                    const uint4 ha = *reinterpret_cast<const uint4 *>(wrow + Fmt<FT>::QH);
                    const uint4 hb = *reinterpret_cast<const uint4 *>(wrow + Fmt<FT>::QH + 16);
                    qh[0] = ha.x; qh[1] = ha.y; qh[2] = ha.z; qh[3] = ha.w;
                    qh[4] = hb.x; qh[5] = hb.y; qh[6] = hb.z; qh[7] = hb.w;
                }
                if (half == 0) dd[(j % SINV) * TM + row] = hdr.x;  // d (low half), dmin (high half)
                uint32_t scp[4], mnp[4];  // (scale, min) of sub-blocks 2t (low byte) and 2t + 1
#pragma unroll
                for (int t = 0; t < 4; t++) scale_min_pair(hdr.y, hdr.z, hdr.w, t, scp[t], mnp[t]);
#pragma unroll
                for (int t = 0; t < 4; t++) {  // unrolled: scp[t] stays in registers
                    const int i = 4 * j + t;
                    if (i >= SA && !warp_wait(bars + EMPTY_A + as, ea_ph, abrt, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();  // the MMAs that read this A slot have completed
                    const uint4 qa = *reinterpret_cast<const uint4 *>(wrow + Fmt<FT>::QS + 32 * t);
                    const uint4 qb = *reinterpret_cast<const uint4 *>(wrow + Fmt<FT>::QS + 16 + 32 * t);
                    if (t == 3) mbar_arrive(bars + EMPTY_W + ws);
                    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    // this half's sub-block: 2t (low nibbles, low scale byte) or 2t + 1
                    const __half sc = __ushort2half_rn((unsigned short)((scp[t] >> (8 * half)) & 255u));
                    const __half2 sc2 = __halves2half2(sc, sc);
                    const __half2 nsc2 = __hmul2(sc2, __float2half2_rn(-1024.0f));
                    const int sh = 4 * half;
                    uint32_t aw[16];  // this half of the step: tensor-memory columns 16 half .. + 15
#pragma unroll
                    for (int cc = 0; cc < 4; cc++) {
                        // columns 8cc .. 8cc+7 of the sub-block: nibbles of bytes 8cc .. 8cc+7
                        uint32_t w0 = q[2 * cc] >> sh, w1 = q[2 * cc + 1] >> sh;
                        if (FT == T_Q5_K) {
                            // the fifth bit of byte l is bit 2t + half of qh[l], moved to bit 4
                            const int hs = 2 * t + half;
                            w0 = (w0 & 0x0F0F0F0Fu) | (((qh[2 * cc] >> hs) & 0x01010101u) << 4);
                            w1 = (w1 & 0x0F0F0F0Fu) | (((qh[2 * cc + 1] >> hs) & 0x01010101u) << 4);
                        }
                        aw[4 * cc] = nib2<FT>(w0, sc2, nsc2);
                        aw[4 * cc + 1] = nib2<FT>(w0 >> 8, sc2, nsc2);
                        aw[4 * cc + 2] = nib2<FT>(w1, sc2, nsc2);
                        aw[4 * cc + 3] = nib2<FT>(w1 >> 8, sc2, nsc2);
                    }
                    tmem_st16(a_lane + (uint32_t)(32 * as + 16 * half), aw);
                    if (t == 0 && half == 0) {
                        // A2 row: the 8 mins of this super-block in natural order, in
                        // chunk 0 (against the hi parts of the sums) and chunk 1 (lo)
                        uint32_t m2[4];
#pragma unroll
                        for (int p = 0; p < 4; p++) {
                            const __half2 h = __halves2half2(__ushort2half_rn((unsigned short)(mnp[p] & 255u)),
                                                             __ushort2half_rn((unsigned short)(mnp[p] >> 8)));
                            m2[p] = *reinterpret_cast<const uint32_t *>(&h);
                        }
                        uint8_t *a2row = sm + OFF_A2 + (j % SA2) * A2_BYTES + row * 16;
                        *reinterpret_cast<uint4 *>(a2row) = make_uint4(m2[0], m2[1], m2[2], m2[3]);
                        *reinterpret_cast<uint4 *>(a2row + TM * 16) = make_uint4(m2[0], m2[1], m2[2], m2[3]);
                        // the generic-proxy writes, seen by the tensor core's async proxy
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    }
                    tc_fence_before();
                    mbar_arrive(bars + FULL_A + as);
                    if (++as == SA) {
                        as = 0;
                        if (i >= SA) ea_ph ^= 1u;
                    }
                }
            }
            if (++ds == a.nsb) {
                ds = 0;
                dT++;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == ISSUER) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)TMEM_COLS)
                     : "memory");
    }
}

// x into the B operands. Block (s, b) stages super-block s of vector b:
// scale = a power of two with max |x piece| * scale < 2^10 (1 for a zero or
// non-finite piece), rows nn = 2b (hi) and 2b + 1 (lo) of the four step
// tiles (b < N / 2), row b of B2 (b < N2: the 32-column sums, hi parts at
// k 0-7, lo parts at k 8-15), and 1 / scale in xinv. Blocks with b >= n
// write the zero rows. 256 threads, thread t = column 256 s + t.
__global__ void __launch_bounds__(256) mm_stage_kernel(const float *x, int n, int K, int N, int N2, uint8_t *xs,
                                                       uint8_t *x2s, float *xinv)
{
    __shared__ float red[8];
    const int s = blockIdx.x, b = blockIdx.y, t = threadIdx.x;  // b < max(N / 2, N2)
    const float xv = b < n ? x[(size_t)b * K + (size_t)s * QK + t] : 0.0f;
    float m = fabsf(xv);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((t & 31) == 0) red[t >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < 8; i++) m = fmaxf(m, red[i]);
    float scale = 1.0f;
    if (m > 0.0f && m <= 3.4e38f) {
        int e = 0;
        frexpf(m, &e);  // m < 2^e
        scale = ldexpf(1.0f, max(-100, min(100, 10 - e)));
    }
    const float v = xv * scale;
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    const int step = t >> 6, chunk = (t >> 3) & 7, e = t & 7;
    if (2 * b < N) {
        uint8_t *run =
            xs + ((size_t)s * 4 + step) * N * 128 + (size_t)chunk * N * 16 + (size_t)(2 * b) * 16 + perm8(e) * 2;
        *reinterpret_cast<__half *>(run) = hi;
        *reinterpret_cast<__half *>(run + 16) = lo;
    }
    // warp w holds sub-block w: its sum, then split
    float sum = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if ((t & 31) == 0 && b < N2) {
        // B2 row b: k 0-7 the hi parts of the 8 sums (chunk 0), k 8-15 the lo parts
        const int j = t >> 5;
        const __half shi = __float2half_rn(sum);
        const __half slo = __float2half_rn(sum - __half2float(shi));
        uint8_t *row = x2s + (size_t)s * N2 * 32 + (size_t)b * 16 + j * 2;
        *reinterpret_cast<__half *>(row) = shi;
        *reinterpret_cast<__half *>(row + (size_t)N2 * 16) = slo;
    }
    if (t == 0 && b < VMAX) xinv[(size_t)s * VMAX + b] = b < n ? 1.0f / scale : 0.0f;
}

// x into the B operands of the Q6_K launch: each 32-column piece of a
// super-block is one step, at k 0-31 and again at k 32-63 (the two parts of
// the split scale multiply the same x). Scale and inverse scale as above;
// no sums (Q6_K has no mins).
__global__ void __launch_bounds__(256) mm_stage6_kernel(const float *x, int n, int K, int N, uint8_t *xs, float *xinv)
{
    __shared__ float red[8];
    const int s = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    const float xv = b < n ? x[(size_t)b * K + (size_t)s * QK + t] : 0.0f;
    float m = fabsf(xv);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((t & 31) == 0) red[t >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < 8; i++) m = fmaxf(m, red[i]);
    float scale = 1.0f;
    if (m > 0.0f && m <= 3.4e38f) {
        int e = 0;
        frexpf(m, &e);  // m < 2^e
        scale = ldexpf(1.0f, max(-100, min(100, 10 - e)));
    }
    const float v = xv * scale;
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    const int step = t >> 5, chunk = (t >> 3) & 3, e = t & 7;
#pragma unroll
    for (int dup = 0; dup < 2; dup++) {
        uint8_t *run = xs + ((size_t)s * 8 + step) * N * 128 + (size_t)(chunk + 4 * dup) * N * 16 + (size_t)(2 * b) * 16 +
                       perm8(e) * 2;
        *reinterpret_cast<__half *>(run) = hi;
        *reinterpret_cast<__half *>(run + 16) = lo;
    }
    if (t == 0) xinv[(size_t)s * VMAX + b] = b < n ? 1.0f / scale : 0.0f;
}

}  // namespace mm
}  // namespace pk

using namespace pk;

namespace {

// cuTensorMapEncodeTiled, from the driver through the runtime (no link
// against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Per-device scratch of gguf_cuda_matmul, grown on demand.
struct MmScratch {
    uint8_t *xs = nullptr, *x2s = nullptr;
    float *xinv = nullptr, *ypart = nullptr;
    unsigned int *arrived = nullptr;
    int *err = nullptr;
    size_t xs_bytes = 0, x2s_bytes = 0, xinv_bytes = 0, ypart_bytes = 0, arrived_bytes = 0;
    int smem_max = 0;
};

int grow(void **p, size_t &have, size_t need, bool zero)
{
    if (have >= need) return 1;
    if (*p) cudaFree(*p);
    *p = nullptr;
    have = 0;
    if (cudaMalloc(p, need) != cudaSuccess) return 0;
    if (zero && cudaMemset(*p, 0, need) != cudaSuccess) return 0;
    have = need;
    return 1;
}

MmScratch *mm_scratch(int dev, size_t xs_b, size_t x2s_b, size_t xinv_b, size_t yp_b, size_t arr_b)
{
    static MmScratch per[64];
    if (dev < 0 || dev >= 64) return nullptr;
    MmScratch &s = per[dev];
    if (!grow((void **)&s.xs, s.xs_bytes, xs_b, false) || !grow((void **)&s.x2s, s.x2s_bytes, x2s_b, false) ||
        !grow((void **)&s.xinv, s.xinv_bytes, xinv_b, false) || !grow((void **)&s.ypart, s.ypart_bytes, yp_b, false) ||
        !grow((void **)&s.arrived, s.arrived_bytes, arr_b, true))
        return nullptr;
    if (s.err == nullptr) {
        if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(s.err, 0, sizeof(int)) != cudaSuccess) return nullptr;
    }
    if (s.smem_max == 0) s.smem_max = pk_mm_smem_max(dev);
    if (s.smem_max == 0) return nullptr;
    return &s;
}

}  // namespace

// The work split of the batched matmul for a matrix of `tiles` row tiles
// and `nsb` super-blocks per row on `sms` SMs: CTAs, and partial slots per
// row tile. At most one CTA per SM, and no more CTAs than split each row
// tile in about four pieces: every CTA pays a fixed cost (tensor memory,
// barriers, the first copies) and the last CTA of a split tile adds the
// pieces up after the others, so short pieces cost more than they save
// (measured on the TinyLlama and Llama shapes: two pieces per tile leave
// SMs idle, eight or one per SM are slower than four).
static void plan_tiles(int tiles, int nsb, int sms, int *ctas, int *maxp)
{
    const long long U = (long long)tiles * nsb;
    long long G = 4LL * tiles;  // about four pieces per tile
    if (G > sms) G = sms;
    if (G > U) G = U;
    int mp = 1;
    for (int T = 0; T < tiles; T++) {
        const int c0 = mm::unit_owner((long long)T * nsb, U, G);
        const int c1 = mm::unit_owner((long long)T * nsb + nsb - 1, U, G);
        if (c1 - c0 + 1 > mp) mp = c1 - c0 + 1;
    }
    *ctas = (int)G;
    *maxp = mp;
}

extern "C" void gguf_cuda_matmul_plan(int rows, int nsb, int sms, int *ctas, int *maxp)
{
    plan_tiles((rows + mm::TM - 1) / mm::TM, nsb, sms, ctas, maxp);
}

// MMA N of the min term: one column per vector, a multiple of 16.
static int mm_n2(int n)
{
    return n <= 16 ? 16 : (n + 15) / 16 * 16;
}

static int mm_sbb(uint32_t type)
{
    return type == T_Q4_K ? mm::Fmt<T_Q4_K>::SBB : type == T_Q5_K ? mm::Fmt<T_Q5_K>::SBB
                                                  : type == T_Q6_K ? mm::Fmt<T_Q6_K>::SBB : 0;
}

static int mm_off_b(uint32_t type)
{
    return type == T_Q5_K ? mm::Lay<T_Q5_K>::OFF_B : type == T_Q6_K ? mm::Lay<T_Q6_K>::OFF_B : mm::Lay<T_Q4_K>::OFF_B;
}

int pk_mm_arena_ok(uint32_t type, uint64_t rows, uint64_t cols, uint64_t row_bytes, const void *data)
{
    if (type != T_Q6_K) return pk_mm_shape_ok(type, rows, cols, row_bytes, data);
    if (cols == 0 || cols % mm::QK || rows == 0 || rows > 0x7FFFFF00ull || cols > 0x7FFFFF00ull) return 0;
    if ((rows + 127) / 128 * (cols / mm::QK) > 0x7FFFFFFFull / 256) return 0;
    return row_bytes == cols / mm::QK * (uint64_t)mm::Fmt<T_Q6_K>::BLK && ((uintptr_t)data & 15) == 0;
}

int pk_mm_shape_ok(uint32_t type, uint64_t rows, uint64_t cols, uint64_t row_bytes, const void *data)
{
    const int sbb = mm_sbb(type);
    if (sbb == 0 || cols == 0 || cols % mm::QK || rows == 0) return 0;
    if (rows > 0x7FFFFF00ull || cols > 0x7FFFFF00ull) return 0;
    if ((rows + 127) / 128 * (cols / mm::QK) > 0x7FFFFFFFull / 256) return 0;  // units and their products fit int
    return row_bytes == cols / mm::QK * (uint64_t)sbb && ((uintptr_t)data & 15) == 0;
}

void pk_mm_need(int rows, int cols, int n, int sms, PkMmNeed *need)
{
    const int nsb = cols / mm::QK, N = (2 * n + 15) / 16 * 16, tiles = (rows + mm::TM - 1) / mm::TM;
    int G = 0, maxp = 0;
    plan_tiles(tiles, nsb, sms, &G, &maxp);
    need->xs = (size_t)nsb * 8 * N * 128;  // 8 steps per super-block (Q6_K; 4 for Q4_K, Q5_K)
    need->x2s = (size_t)nsb * N * 32;
    need->xinv = (size_t)nsb * mm::VMAX * 4;
    need->ypart = (size_t)tiles * maxp * n * mm::TM * sizeof(float);
    need->arrived = (size_t)tiles * mm::DQ_WARPS * sizeof(unsigned);
}

int pk_mm_smem_max(int dev)
{
    static int per[64] = {0};
    if (dev < 0 || dev >= 64) return 0;
    if (per[dev] == 0) {
        int optin = 0;
        cudaFuncAttributes fa, fb, fc;
        if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            cudaFuncGetAttributes(&fa, mm::qk_mm_kernel<T_Q4_K>) != cudaSuccess ||
            cudaFuncGetAttributes(&fb, mm::qk_mm_kernel<T_Q5_K>) != cudaSuccess ||
            cudaFuncGetAttributes(&fc, mm::qk_mm_kernel<T_Q6_K>) != cudaSuccess)
            return 0;
        size_t stat = fa.sharedSizeBytes;
        if (fb.sharedSizeBytes > stat) stat = fb.sharedSizeBytes;
        if (fc.sharedSizeBytes > stat) stat = fc.sharedSizeBytes;
        const int avail = optin - (int)stat;
        if (avail < mm::Lay<T_Q5_K>::OFF_B + 3 * mm::B_SLOT_MAX + 128 ||
            avail < mm::Lay<T_Q4_K>::OFF_B + 3 * mm::B_SLOT_MAX + 128 ||
            avail < mm::Lay<T_Q6_K>::OFF_B + 3 * mm::B_SLOT_MAX + 128)
            return 0;
        if (cudaFuncSetAttribute(mm::qk_mm_kernel<T_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, avail) !=
                cudaSuccess ||
            cudaFuncSetAttribute(mm::qk_mm_kernel<T_Q5_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, avail) !=
                cudaSuccess ||
            cudaFuncSetAttribute(mm::qk_mm_kernel<T_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, avail) !=
                cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        per[dev] = avail;
    }
    return per[dev];
}

int pk_mm_stage(uint32_t type, const float *x, int n, int cols, const PkMmScratch *s, cudaStream_t st)
{
    if (n < 1 || n > mm::VMAX || s == nullptr) return 0;
    const int N = (2 * n + 15) / 16 * 16;
    if (type == T_Q6_K) {
        mm::mm_stage6_kernel<<<dim3(cols / mm::QK, N / 2), 256, 0, st>>>(x, n, cols, N, s->xs, s->xinv);
    } else {
        const int N2 = mm_n2(n);
        mm::mm_stage_kernel<<<dim3(cols / mm::QK, N / 2 > N2 ? N / 2 : N2), 256, 0, st>>>(x, n, cols, N, N2, s->xs,
                                                                                         s->x2s, s->xinv);
    }
    return cudaGetLastError() == cudaSuccess;
}

int pk_mm_run_staged(const PkMmSeg *seg, int nseg, int cols, int n, const PkMmScratch *s, int sms, cudaStream_t st)
{
    if (n < 1 || n > mm::VMAX || s == nullptr || s->smem_max <= 0 || nseg < 1 || nseg > mm::MSEG) return 0;
    const uint32_t type = seg[0].type;
    const int sbb = mm_sbb(type), off_b = mm_off_b(type);
    if (sbb == 0) return 0;
    for (int i = 1; i < nseg; i++)
        if (seg[i].type != type) return 0;  // one format per launch
    const int nsb = cols / mm::QK;
    const int N = (2 * n + 15) / 16 * 16;
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_tiled();
    if (enc == nullptr && type != T_Q6_K) return 0;
    mm::MmMaps maps;
    memset(&maps, 0, sizeof(maps));
    mm::MmArgs a;
    memset(&a, 0, sizeof(a));
    a.nseg = nseg;
    int tiles = 0;
    for (int i = 0; i < nseg; i++) {
        a.seg_w[i] = seg[i].w;
        a.seg_rb[i] = seg[i].row_bytes;
        a.tile0[i] = tiles;
        a.seg_rows[i] = seg[i].rows;
        a.seg_y[i] = seg[i].y;
        tiles += (seg[i].rows + mm::TM - 1) / mm::TM;
        if (type == T_Q6_K) continue;  // each row's window by a bulk copy: no tensor map
        const cuuint64_t gdim[2] = {(cuuint64_t)seg[i].row_bytes, (cuuint64_t)seg[i].rows};
        const cuuint64_t gstride[1] = {(cuuint64_t)seg[i].row_bytes};
        const cuuint32_t box[2] = {(cuuint32_t)sbb, (cuuint32_t)mm::TM};
        const cuuint32_t estride[2] = {1, 1};
        if (enc(&maps.m[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(seg[i].w), gdim, gstride, box,
                estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return 0;
    }
    for (int i = nseg; i <= mm::MSEG; i++) a.tile0[i] = tiles;
    int G = 0, maxp = 0;
    plan_tiles(tiles, nsb, sms, &G, &maxp);
    a.nsb = nsb;
    a.xs = s->xs;
    a.x2s = s->x2s;
    a.xinv = s->xinv;
    a.n = n;
    a.N = N;
    a.N2 = mm_n2(n);
    a.b_slot = N * 128 + (type == T_Q6_K ? 0 : a.N2 * 32);
    a.sb = (s->smem_max - off_b - 128) / a.b_slot;
    if (a.sb > mm::SB_MAX) a.sb = mm::SB_MAX;
    a.U = tiles * nsb;
    a.G = G;
    a.maxp = maxp;
    a.ypart = s->ypart;
    a.arrived = s->arrived;
    a.err = s->err;
    // one CTA per SM: each allocates all 512 tensor-memory columns
    int smem = off_b + a.sb * a.b_slot + 128;
    if (smem <= s->smem_max / 2) smem = s->smem_max / 2 + 128;
    if (type == T_Q5_K) {
        mm::qk_mm_kernel<T_Q5_K><<<G, mm::THREADS, smem, st>>>(maps, a);
    } else if (type == T_Q6_K) {
        mm::qk_mm_kernel<T_Q6_K><<<G, mm::THREADS, smem, st>>>(maps, a);
    } else {
        mm::qk_mm_kernel<T_Q4_K><<<G, mm::THREADS, smem, st>>>(maps, a);
    }
    return cudaGetLastError() == cudaSuccess;
}

int pk_mm_run(uint32_t type, const uint8_t *w, uint64_t row_bytes, int rows, int cols, const float *x, int n,
              float *y, const PkMmScratch *s, int sms, cudaStream_t st)
{
    PkMmSeg seg;
    seg.type = type;
    seg.w = w;
    seg.row_bytes = row_bytes;
    seg.rows = rows;
    seg.y = y;
    return pk_mm_stage(type, x, n, cols, s, st) && pk_mm_run_staged(&seg, 1, cols, n, s, sms, st);
}

extern "C" int gguf_cuda_matmul(const GGUFWeight *w, const float *x, int n, float *y, void *stream)
{
    if (w == nullptr || w->data == nullptr || x == nullptr || y == nullptr || n < 1 || n > mm::VMAX) return 0;
    if (!pk_mm_shape_ok(w->type, w->rows, w->cols, w->row_bytes, w->data)) return 0;
    const int rows = (int)w->rows, K = (int)w->cols;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return 0;
    PkMmNeed need;
    pk_mm_need(rows, K, n, sms, &need);
    MmScratch *s = mm_scratch(dev, need.xs, need.x2s, need.xinv, need.ypart, need.arrived);
    if (s == nullptr) return 0;
    PkMmScratch sc;
    sc.xs = s->xs;
    sc.x2s = s->x2s;
    sc.xinv = s->xinv;
    sc.ypart = s->ypart;
    sc.arrived = s->arrived;
    sc.err = s->err;
    sc.smem_max = s->smem_max;
    return pk_mm_run(w->type, (const uint8_t *)w->data, w->row_bytes, rows, K, x, n, y, &sc, sms,
                     (cudaStream_t)stream);
}

// Error word of gguf_cuda_matmul on the current device (0: no wait has run
// out of time), cleared by the read; -1 when it cannot be read.
extern "C" int gguf_cuda_matmul_error(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    MmScratch *s = mm_scratch(dev, 0, 0, 0, 0, 0);
    if (s == nullptr) return -1;
    int v = 0;
    if (cudaMemcpy(&v, s->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v != 0) {
        // an aborted call can leave tile counters behind: clear them
        if (cudaMemset(s->err, 0, sizeof(int)) != cudaSuccess) return -1;
        if (s->arrived != nullptr && cudaMemset(s->arrived, 0, s->arrived_bytes) != cudaSuccess) return -1;
    }
    return v;
}
