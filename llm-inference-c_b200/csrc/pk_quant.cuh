// pk_quant.cuh - device-side GGUF block formats for sm_100a.
//
// Two families of functions:
//   * decode_elem<T>(): one weight of a block to FP32, bit-identical to the
//     reference decoders (src/gguf_quant.c:92-345). Every product/difference
//     uses the explicitly rounded intrinsics (__fmul_rn, __fsub_rn) so nvcc
//     cannot contract them into FMAs; the reference is compiled with
//     -std=c11, i.e. -ffp-contract=off.
//   * unit_*(): the fused dequant-dot of one 64-column "unit" of a row with
//     the unit's activations held in registers in integer form (XUnit). This
//     is the hot loop of every matvec. It follows the reference's algebra
//     (src/gguf_model.c:445-691): per 32- or 16-weight group, sum q*x first
//     and apply the group scale (and, for Q4_K/Q5_K, subtract
//     dmin*m*sum(x)) once per group. The group sums are exact integer dp4a
//     sums over a 23-bit fixed-point copy of x, so results agree with the
//     reference's float32 kernels to ~1e-7 relative, not bit for bit.
//
// Units (64 consecutive columns each, so activation slices are shared by
// every format):
//   Q4_K / Q5_K : block u/4, sub-block pair j = u%4 (weights 64j..64j+63)
//   Q6_K        : block u/4, half h = (u%4)/2, nibble half mm = u%2
//                 (weights 128h + 64mm .. +63)
//   Q4_0 / Q8_0 : blocks 2u and 2u+1 (the second may be absent)
//   F32 / F16   : columns 64u .. 64u+63 (guarded at the row end)
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

namespace pk {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

__host__ __device__ inline int block_weights(int t)
{
    return (t == T_Q4_0 || t == T_Q8_0) ? 32 : (t == T_F32 || t == T_F16) ? 1 : 256;
}
__host__ __device__ inline int block_bytes(int t)
{
    switch (t) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q4_0: return 18;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    default: return 0;
    }
}

// Exact IEEE half -> float for all 65536 inputs (subnormals normalised,
// inf/NaN keep their payload), matching src/gguf_quant.c:6-59.
__device__ __forceinline__ float h2f(uint32_t h)
{
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 1023u;
    uint32_t bits;
    if (e == 31u) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0u) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0u) {
        bits = sign;
    } else {
        uint32_t n = __clz(m) - 21u;  // shifts that bring the leading one to bit 10
        bits = sign | ((113u - n) << 23) | (((m << n) & 1023u) << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

// 6-bit (scale, min) pair i of the 12 packed scale bytes
// (src/gguf_quant.c:65-90).
__device__ __forceinline__ void scale_min(const uint8_t *s, int i, uint32_t &sc, uint32_t &mn)
{
    if (i < 4) {
        sc = s[i] & 63u;
        mn = s[i + 4] & 63u;
    } else {
        sc = (s[i + 4] & 15u) | ((uint32_t)(s[i - 4] >> 6) << 4);
        mn = (uint32_t)(s[i + 4] >> 4) | ((uint32_t)(s[i] >> 6) << 4);
    }
}

// Same, from the 12 scale bytes held in three 32-bit words.
__device__ __forceinline__ void scale_min_w(uint32_t s0, uint32_t s1, uint32_t s2, int i,
                                            uint32_t &sc, uint32_t &mn)
{
    // byte k of the 12: word k/4, shift 8*(k%4)
    auto B = [&](int k) -> uint32_t {
        uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
        return (w >> (8 * (k & 3))) & 255u;
    };
    if (i < 4) {
        sc = B(i) & 63u;
        mn = B(i + 4) & 63u;
    } else {
        sc = (B(i + 4) & 15u) | ((B(i - 4) >> 6) << 4);
        mn = (B(i + 4) >> 4) | ((B(i) >> 6) << 4);
    }
}

// ------------------------------------------------------------------ //
// Bit-exact single-weight decoders                                   //
// ------------------------------------------------------------------ //

// Weight `i` (0..255 or 0..31) of the block at `b`.
template <int T>
__device__ __forceinline__ float decode_elem(const uint8_t *b, int i);

template <>
__device__ __forceinline__ float decode_elem<T_Q4_K>(const uint8_t *b, int i)
{
    const float d = h2f(ld_u16(b)), dmin = h2f(ld_u16(b + 2));
    const int j = i >> 6, hi = (i >> 5) & 1, l = i & 31;
    uint32_t sc, mn;
    scale_min(b + 4, 2 * j + hi, sc, mn);
    const uint32_t byte = b[16 + 32 * j + l];
    const uint32_t q = hi ? (byte >> 4) : (byte & 15u);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
}

template <>
__device__ __forceinline__ float decode_elem<T_Q5_K>(const uint8_t *b, int i)
{
    const float d = h2f(ld_u16(b)), dmin = h2f(ld_u16(b + 2));
    const int j = i >> 6, hi = (i >> 5) & 1, l = i & 31;
    uint32_t sc, mn;
    scale_min(b + 4, 2 * j + hi, sc, mn);
    const uint32_t byte = b[48 + 32 * j + l];
    const uint32_t bit = (b[16 + l] >> (2 * j + hi)) & 1u;
    const uint32_t q = (hi ? (byte >> 4) : (byte & 15u)) + (bit << 4);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
}

template <>
__device__ __forceinline__ float decode_elem<T_Q6_K>(const uint8_t *b, int i)
{
    const int h = i >> 7, r = i & 127, m = r >> 5, l = r & 31;
    const uint32_t qlb = b[64 * h + l + 32 * (m & 1)];
    const uint32_t nib = (m >= 2) ? (qlb >> 4) : (qlb & 15u);
    const uint32_t hb = (b[128 + 32 * h + l] >> (2 * m)) & 3u;
    const int q = (int)(nib | (hb << 4)) - 32;
    const float d = h2f(ld_u16(b + 208));
    const float sc = (float)(int8_t)b[192 + (i >> 4)];
    return __fmul_rn(__fmul_rn(d, sc), (float)q);
}

template <>
__device__ __forceinline__ float decode_elem<T_Q4_0>(const uint8_t *b, int i)
{
    const float d = h2f(ld_u16(b));
    const uint32_t byte = b[2 + (i & 15)];
    const int q = (int)(i < 16 ? (byte & 15u) : (byte >> 4)) - 8;
    return __fmul_rn(d, (float)q);
}

template <>
__device__ __forceinline__ float decode_elem<T_Q8_0>(const uint8_t *b, int i)
{
    return __fmul_rn((float)(int8_t)b[2 + i], h2f(ld_u16(b)));
}

template <>
__device__ __forceinline__ float decode_elem<T_F32>(const uint8_t *b, int i)
{
    uint32_t v = (uint32_t)b[4 * i] | ((uint32_t)b[4 * i + 1] << 8) | ((uint32_t)b[4 * i + 2] << 16) |
                 ((uint32_t)b[4 * i + 3] << 24);
    return __uint_as_float(v);
}

template <>
__device__ __forceinline__ float decode_elem<T_F16>(const uint8_t *b, int i)
{
    return h2f(ld_u16(b + 2 * i));
}

// Column `c` of a row of type t (runtime dispatch).
__device__ __forceinline__ float decode_col(int t, const uint8_t *row, int c)
{
    switch (t) {
    case T_Q4_K: return decode_elem<T_Q4_K>(row + (c >> 8) * 144, c & 255);
    case T_Q5_K: return decode_elem<T_Q5_K>(row + (c >> 8) * 176, c & 255);
    case T_Q6_K: return decode_elem<T_Q6_K>(row + (c >> 8) * 210, c & 255);
    case T_Q4_0: return decode_elem<T_Q4_0>(row + (c >> 5) * 18, c & 31);
    case T_Q8_0: return decode_elem<T_Q8_0>(row + (c >> 5) * 34, c & 31);
    case T_F32: return decode_elem<T_F32>(row, c);
    case T_F16: return decode_elem<T_F16>(row, c);
    default: return __int_as_float(0x7FC00000);
    }
}

// decode_col as a real call: for the cold paths of the decode step (the
// embedding row of layer 0), where inlining all seven decoders at every
// use would only bloat the hot kernel's code.
static __device__ __noinline__ float decode_col_call(int t, const uint8_t *row, int c)
{
    return decode_col(t, row, c);
}

// ------------------------------------------------------------------ //
// Fused dequant-dot of one 64-column unit                            //
// ------------------------------------------------------------------ //

// ------------------------------------------------------------------ //
// Integer form of the activations                                    //
// ------------------------------------------------------------------ //
//
// Before a matvec every 32-column group g of x is written as
//     x_i = s_g * (d0_i + 2^8 d1_i + 2^16 d2_i),   s_g = 2^(E_g - 22)
// with E_g the binary exponent of max|x_g| and d0..d2 signed bytes: a 23-bit
// fixed-point copy of x (relative error <= 2^-23 of the group maximum). The
// dot of a group with integer quants q is then three exact int32 dp4a sums,
// one per digit plane, combined in float once per group:
//     sum_i q_i x_i = s_g * (A0 + 2^8 A1 + 2^16 A2),  A_p = sum_i q_i dp_i.
// One dp4a does four multiply-adds, so a weight costs ~3/4 dp4a plus its
// share of the nibble unpack, instead of an int->float conversion and an FMA.
// The group scales of the formats are applied afterwards exactly as the
// reference's fast kernels do (src/gguf_model.c:445-691).

// Shared-memory layout per 64-column unit u (two groups 2u, 2u+1):
//   digits : 208 bytes at u*208: [group][plane][32 bytes] + 16 pad
//   info   : 80 bytes at u*80:   per group {scale, sum(x), dsum[half][plane]}
//            (8 words each) + 16 pad. dsum are the digit sums of each
//            16-column half, used to apply q - 32 / q - 8 offsets.
constexpr int XQ_UNIT_BYTES = 208;
constexpr int XG_UNIT_WORDS = 20;

struct XUnit {
    uint32_t d[2][3][8];  // digit words: bytes of columns 4w..4w+3
    float scale[2];
    float sum[2];
    int dsum[2][2][3];    // [group][half][plane]
};

__device__ __forceinline__ void load_xunit(const uint8_t *xq, const float *xg, int u, XUnit &x)
{
    const uint4 *q = reinterpret_cast<const uint4 *>(xq + u * XQ_UNIT_BYTES);
    uint32_t *dst = &x.d[0][0][0];
#pragma unroll
    for (int i = 0; i < 12; i++) {
        const uint4 t = q[i];
        dst[4 * i] = t.x;
        dst[4 * i + 1] = t.y;
        dst[4 * i + 2] = t.z;
        dst[4 * i + 3] = t.w;
    }
    const float4 *gp = reinterpret_cast<const float4 *>(xg + u * XG_UNIT_WORDS);
#pragma unroll
    for (int g = 0; g < 2; g++) {
        const float4 a = gp[2 * g], b = gp[2 * g + 1];
        x.scale[g] = a.x;
        x.sum[g] = a.y;
        x.dsum[g][0][0] = __float_as_int(a.z);
        x.dsum[g][0][1] = __float_as_int(a.w);
        x.dsum[g][0][2] = __float_as_int(b.x);
        x.dsum[g][1][0] = __float_as_int(b.y);
        x.dsum[g][1][1] = __float_as_int(b.z);
        x.dsum[g][1][2] = __float_as_int(b.w);
    }
}

// Four unsigned bytes of a times four signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)
{
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// Four signed bytes of a times four signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c)
{
    int r;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ float planes(int a0, int a1, int a2)
{
    // a0 + 2^8 a1 is exact in int32 (|a1| < 2^23); two conversions, one FMA.
    return fmaf((float)a2, 65536.0f, (float)(a0 + (a1 << 8)));
}

// fp16 -> fp32 by the hardware conversion: exact for every finite value,
// which is all a matvec needs (a NaN scale gives a NaN either way).
__device__ __forceinline__ float hf(uint32_t bits16)
{
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

// Byte b of w as a float, exactly: the byte goes into the mantissa of
// 2^23 (one byte permute) and 2^23 is subtracted (one add), which avoids
// the slower integer-to-float conversion.
__device__ __forceinline__ float byte_f(uint32_t w, int b)
{
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)b)) - 8388608.0f;
}

// The two 6-bit (scale, min) pairs of sub-blocks 2j and 2j+1 of a Q4_K /
// Q5_K block, from the scale bytes held in three words s0 = bytes 0..3,
// s1 = 4..7, s2 = 8..11 (src/gguf_quant.c:65-90): pairs come out packed as
// two bytes (sub-block 2j in the low byte).
__device__ __forceinline__ void scale_min_pair(uint32_t s0, uint32_t s1, uint32_t s2, int j, uint32_t &sc,
                                               uint32_t &mn)
{
    const int sh = 16 * (j & 1);
    const uint32_t a = (s0 >> sh) & 0xFFFFu, b = (s1 >> sh) & 0xFFFFu, c = (s2 >> sh) & 0xFFFFu;
    const uint32_t sc_lo = a & 0x3F3Fu, mn_lo = b & 0x3F3Fu;
    const uint32_t sc_hi = (c & 0x0F0Fu) | (((a >> 6) & 0x0303u) << 4);
    const uint32_t mn_hi = ((c >> 4) & 0x0F0Fu) | (((b >> 6) & 0x0303u) << 4);
    sc = j < 2 ? sc_lo : sc_hi;
    mn = j < 2 ? mn_lo : mn_hi;
}

// NW consecutive 32-bit words starting at a 2-byte-aligned shared address
// (rows of Q6_K / Q4_0 / Q8_0 are not 4-byte aligned in general).
template <int NW>
__device__ __forceinline__ void ld_words_a2(const uint8_t *p, uint32_t *w)
{
    const uintptr_t a = (uintptr_t)p;
    const uint32_t *base = (const uint32_t *)(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3) * 8u;  // 0 or 16
    uint32_t prev = base[0];
#pragma unroll
    for (int k = 0; k < NW; k++) {
        const uint32_t next = base[k + 1];
        w[k] = __funnelshift_r(prev, next, sh);
        prev = next;
    }
}

// ------------------------------------------------------------------ //
// Fused dequant-dot of one 64-column unit                            //
// ------------------------------------------------------------------ //

// Q4_K unit: d*sc*sum(q*x) - dmin*m*sum(x) for sub-blocks 2j and 2j+1
// (src/gguf_model.c:457-507). `row` is 16-byte aligned (144 = 9*16). High
// nibbles enter dp4a unshifted (16 q), and the 1/16 folds into the float
// combine, exactly.
__device__ __forceinline__ float unit_q4k(const uint8_t *row, int u, const XUnit &x)
{
    const uint8_t *blk = row + (u >> 2) * 144;
    const int j = u & 3;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * j);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int A[2][3] = {{0, 0, 0}, {0, 0, 0}};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t lo = w[k] & 0x0F0F0F0Fu, hi16 = w[k] & 0xF0F0F0F0u;
#pragma unroll
        for (int p = 0; p < 3; p++) {
            A[0][p] = dp4a_us(lo, x.d[0][p][k], A[0][p]);
            A[1][p] = dp4a_us(hi16, x.d[1][p][k], A[1][p]);
        }
    }
    uint32_t sc, mn;
    scale_min_pair(hdr.y, hdr.z, hdr.w, j, sc, mn);
    const float d = hf(hdr.x & 0xFFFFu), dmin = hf(hdr.x >> 16);
    const float s0v = x.scale[0] * planes(A[0][0], A[0][1], A[0][2]);
    const float s1v = (x.scale[1] * 0.0625f) * planes(A[1][0], A[1][1], A[1][2]);
    const float ds = fmaf(byte_f(sc, 1), s1v, byte_f(sc, 0) * s0v);
    const float dm = fmaf(byte_f(mn, 1), x.sum[1], byte_f(mn, 0) * x.sum[0]);
    return fmaf(d, ds, -dmin * dm);
}

// Q5_K unit: as Q4_K with the fifth bit from qh (bits 2j, 2j+1),
// src/gguf_model.c:574-626.
__device__ __forceinline__ float unit_q5k(const uint8_t *row, int u, const XUnit &x)
{
    const uint8_t *blk = row + (u >> 2) * 176;
    const int j = u & 3;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 ha = *reinterpret_cast<const uint4 *>(blk + 16);
    const uint4 hb = *reinterpret_cast<const uint4 *>(blk + 32);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * j);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint32_t h[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    int A[2][3] = {{0, 0, 0}, {0, 0, 0}};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t lo = (w[k] & 0x0F0F0F0Fu) | (((h[k] >> (2 * j)) & 0x01010101u) << 4);
        const uint32_t hi = ((w[k] >> 4) & 0x0F0F0F0Fu) | (((h[k] >> (2 * j + 1)) & 0x01010101u) << 4);
#pragma unroll
        for (int p = 0; p < 3; p++) {
            A[0][p] = dp4a_us(lo, x.d[0][p][k], A[0][p]);
            A[1][p] = dp4a_us(hi, x.d[1][p][k], A[1][p]);
        }
    }
    uint32_t sc, mn;
    scale_min_pair(hdr.y, hdr.z, hdr.w, j, sc, mn);
    const float d = hf(hdr.x & 0xFFFFu), dmin = hf(hdr.x >> 16);
    const float s0v = x.scale[0] * planes(A[0][0], A[0][1], A[0][2]);
    const float s1v = x.scale[1] * planes(A[1][0], A[1][1], A[1][2]);
    const float ds = fmaf(byte_f(sc, 1), s1v, byte_f(sc, 0) * s0v);
    const float dm = fmaf(byte_f(mn, 1), x.sum[1], byte_f(mn, 0) * x.sum[0]);
    return fmaf(d, ds, -dmin * dm);
}

// Q6_K unit: columns 128h + 64mm + [0, 64) of block u/4. Weight
// 128h + 64mm + 32k + l uses ql[64h + 32k + l] (low nibble if mm = 0, high
// if mm = 1) and bits 2(2mm + k) of qh[32h + l]; (q - 32) times the int8
// scale of its 16-weight group, times d (src/gguf_model.c:516-566).
__device__ __forceinline__ float unit_q6k(const uint8_t *row, int u, const XUnit &x)
{
    const uint8_t *blk = row + (u >> 2) * 210;
    const int h = (u >> 1) & 1, mm = u & 1;
    uint32_t ql[16], qh[8];
    ld_words_a2<16>(blk + 64 * h, ql);
    ld_words_a2<8>(blk + 128 + 32 * h, qh);
    int A[4][3];
#pragma unroll
    for (int i = 0; i < 4; i++) A[i][0] = A[i][1] = A[i][2] = 0;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int sh = 2 * (2 * mm + k);
#pragma unroll
        for (int wv = 0; wv < 8; wv++) {
            const uint32_t nib = mm ? ((ql[8 * k + wv] >> 4) & 0x0F0F0F0Fu) : (ql[8 * k + wv] & 0x0F0F0F0Fu);
            const uint32_t q6 = nib | (((qh[wv] >> sh) & 0x03030303u) << 4);
            const int g16 = 2 * k + (wv >> 2);
#pragma unroll
            for (int p = 0; p < 3; p++) A[g16][p] = dp4a_us(q6, x.d[k][p][wv], A[g16][p]);
        }
    }
    const float d = hf(ld_u16(blk + 208));
    // the four int8 scales of these 64 weights, biased to unsigned bytes
    const uint8_t *scp = blk + 192 + 8 * h + 4 * mm;
    const uint32_t scw = (ld_u16(scp) | (ld_u16(scp + 2) << 16)) ^ 0x80808080u;
    float total = 0.0f;
#pragma unroll
    for (int g16 = 0; g16 < 4; g16++) {
        const int g = g16 >> 1, half = g16 & 1;
        const float v = x.scale[g] * planes(A[g16][0] - 32 * x.dsum[g][half][0], A[g16][1] - 32 * x.dsum[g][half][1],
                                            A[g16][2] - 32 * x.dsum[g][half][2]);
        // byte + 128 as a float, minus 128: the signed scale, exactly
        const float scf = __uint_as_float(__byte_perm(scw, 0x4B000000u, 0x7440u | (uint32_t)g16)) - 8388736.0f;
        total = fmaf(d * scf, v, total);
    }
    return total;
}

// Q4_0 unit: blocks 2u and (if present) 2u+1, w = d*(q-8),
// src/gguf_model.c:633-661.
__device__ __forceinline__ float unit_q4_0(const uint8_t *row, int u, int nblocks, const XUnit &x)
{
    float total = 0.0f;
#pragma unroll
    for (int kb = 0; kb < 2; kb++) {
        if (2 * u + kb < nblocks) {
            const uint8_t *blk = row + (2 * u + kb) * 18;
            uint32_t w[4];
            ld_words_a2<4>(blk + 2, w);
            int A[3] = {0, 0, 0};
#pragma unroll
            for (int wv = 0; wv < 4; wv++) {
                const uint32_t lo = w[wv] & 0x0F0F0F0Fu, hi = (w[wv] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    A[p] = dp4a_us(lo, x.d[kb][p][wv], A[p]);
                    A[p] = dp4a_us(hi, x.d[kb][p][4 + wv], A[p]);
                }
            }
            const float v = x.scale[kb] * planes(A[0] - 8 * (x.dsum[kb][0][0] + x.dsum[kb][1][0]),
                                                 A[1] - 8 * (x.dsum[kb][0][1] + x.dsum[kb][1][1]),
                                                 A[2] - 8 * (x.dsum[kb][0][2] + x.dsum[kb][1][2]));
            total = fmaf(hf(ld_u16(blk)), v, total);
        }
    }
    return total;
}

// Q8_0 unit: blocks 2u and (if present) 2u+1, w = q*d,
// src/gguf_model.c:664-691.
__device__ __forceinline__ float unit_q8_0(const uint8_t *row, int u, int nblocks, const XUnit &x)
{
    float total = 0.0f;
#pragma unroll
    for (int kb = 0; kb < 2; kb++) {
        if (2 * u + kb < nblocks) {
            const uint8_t *blk = row + (2 * u + kb) * 34;
            uint32_t w[8];
            ld_words_a2<8>(blk + 2, w);
            int A[3] = {0, 0, 0};
#pragma unroll
            for (int wv = 0; wv < 8; wv++) {
#pragma unroll
                for (int p = 0; p < 3; p++) A[p] = dp4a_ss(w[wv], x.d[kb][p][wv], A[p]);
            }
            total = fmaf(hf(ld_u16(blk)), x.scale[kb] * planes(A[0], A[1], A[2]), total);
        }
    }
    return total;
}

// F32 / F16 unit: columns 64u .. min(64u+64, cols). The activations are
// rebuilt from the digits in shared memory (these formats are rare in the
// quantized path, so they do not get a register copy).
__device__ __forceinline__ float unit_float(int t, const uint8_t *row, int u, int cols, const uint8_t *xq,
                                            const float *xg)
{
    float s = 0.0f;
    const int8_t *dq = reinterpret_cast<const int8_t *>(xq + u * XQ_UNIT_BYTES);
#pragma unroll 4
    for (int i = 0; i < 64; i++) {
        const int c = 64 * u + i;
        if (c < cols) {
            const int g = i >> 5, l = i & 31;
            const float xv = xg[u * XG_UNIT_WORDS + 8 * g] *
                             planes(dq[96 * g + l], dq[96 * g + 32 + l], dq[96 * g + 64 + l]);
            const float wv = t == T_F32 ? decode_elem<T_F32>(row, c) : decode_elem<T_F16>(row, c);
            s = fmaf(wv, xv, s);
        }
    }
    return s;
}

// ------------------------------------------------------------------ //
// KV cache entries: float, or IEEE half (round to nearest even on the //
// append, exact widening on the read)                                //
// ------------------------------------------------------------------ //

__device__ __forceinline__ float kv_load(const float *p, size_t i)
{
    return p[i];
}
__device__ __forceinline__ float kv_load(const __half *p, size_t i)
{
    return __half2float(p[i]);
}
__device__ __forceinline__ void kv_store(float *p, size_t i, float v)
{
    p[i] = v;
}
__device__ __forceinline__ void kv_store(__half *p, size_t i, float v)
{
    p[i] = __float2half_rn(v);
}
// The value an entry holds once stored.
__device__ __forceinline__ float kv_round(const float *, float v)
{
    return v;
}
__device__ __forceinline__ float kv_round(const __half *, float v)
{
    return __half2float(__float2half_rn(v));
}
// Entries i .. i+3 (i a multiple of 4) as a float4: one 16- or 8-byte load.
__device__ __forceinline__ float4 kv_load4(const float *p, size_t i)
{
    return *reinterpret_cast<const float4 *>(p + i);
}
__device__ __forceinline__ float4 kv_load4(const __half *p, size_t i)
{
    const uint2 u = *reinterpret_cast<const uint2 *>(p + i);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// Host: copy n float entries into a KV cache at entry offset `off`, as the
// cache holds them (float, or IEEE half rounded to nearest even), on `st`,
// then wait. Returns the CUDA error.
static inline cudaError_t kv_upload(void *cache, int half, size_t off, const float *src, size_t n, cudaStream_t st)
{
    if (!half) {
        cudaError_t e = cudaMemcpyAsync(static_cast<float *>(cache) + off, src, n * sizeof(float),
                                        cudaMemcpyHostToDevice, st);
        return e != cudaSuccess ? e : cudaStreamSynchronize(st);
    }
    __half *h = static_cast<__half *>(malloc(n * sizeof(__half)));
    if (h == nullptr) return cudaErrorMemoryAllocation;
    for (size_t i = 0; i < n; i++) h[i] = __float2half_rn(src[i]);
    cudaError_t e = cudaMemcpyAsync(static_cast<__half *>(cache) + off, h, n * sizeof(__half),
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    free(h);
    return e;
}

}  // namespace pk
