// pk_quant.cuh - device-side GGUF block formats for sm_100a.
//
// Two families of functions:
//   * decode_elem<T>(): one weight of a block to FP32, bit-identical to the
//     reference decoders (src/gguf_quant.c:92-345). Every product/difference
//     uses the explicitly rounded intrinsics (__fmul_rn, __fsub_rn) so nvcc
//     cannot contract them into FMAs; the reference is compiled with
//     -std=c11, i.e. -ffp-contract=off.
//   * unit_dot<T>(): the fused dequant-dot of one 64-column "unit" of a row
//     with 64 activations held in registers. This is the hot loop of every
//     matvec. It follows the reference's algebra (src/gguf_model.c:445-691):
//     per 32- or 16-weight group, sum q*x first and apply the group scale
//     (and, for Q4_K/Q5_K, subtract dmin*m*sum(x)) once per group. The sums
//     use FMA accumulation instead of the reference's pairwise trees, so
//     results agree to float32 rounding (~1e-7 relative), not bit for bit.
//
// Units (64 consecutive columns each, so activation slices are shared by
// every format):
//   Q4_K / Q5_K : block u/4, sub-block pair j = u%4 (weights 64j..64j+63)
//   Q6_K        : block u/4, half h = (u%4)/2, nibble half mm = u%2
//                 (weights 128h + 64mm .. +63)
//   Q4_0 / Q8_0 : blocks 2u and 2u+1 (the second may be absent)
//   F32 / F16   : columns 64u .. 64u+63 (guarded at the row end)
#pragma once
#include <stdint.h>

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

// ------------------------------------------------------------------ //
// Fused dequant-dot of one 64-column unit                            //
// ------------------------------------------------------------------ //

// 2^23 + n as a float for a small integer n, then minus 2^23: an exact
// int->float conversion in two cheap ALU ops (avoids the slow I2F path).
__device__ __forceinline__ float u2f_small(uint32_t n)
{
    return __uint_as_float(0x4B000000u | n) - 8388608.0f;
}

// Four consecutive 32-bit words starting at a 2-byte-aligned shared
// address (rows of Q6_K / Q4_0 / Q8_0 are not 4-byte aligned in general).
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

// Q4_K unit: d*sc*sum(q*x) - dmin*m*sum(x) for sub-blocks 2j and 2j+1.
// `row` is 16-byte aligned (Q4_K rows are multiples of 144 = 9*16 bytes).
__device__ __forceinline__ float unit_q4k(const uint8_t *row, int u, const float *xr, float xs_lo,
                                          float xs_hi)
{
    const uint8_t *blk = row + (u >> 2) * 144;
    const int j = u & 3;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * j);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    float slo = 0.0f, shi = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
#pragma unroll
        for (int b = 0; b < 4; b++) {
            slo = fmaf(u2f_small((w[k] >> (8 * b)) & 15u), xr[4 * k + b], slo);
            shi = fmaf(u2f_small((w[k] >> (8 * b + 4)) & 15u), xr[32 + 4 * k + b], shi);
        }
    }
    const float d = h2f(hdr.x & 0xFFFFu), dmin = h2f(hdr.x >> 16);
    uint32_t s0, m0, s1, m1;
    scale_min_w(hdr.y, hdr.z, hdr.w, 2 * j, s0, m0);
    scale_min_w(hdr.y, hdr.z, hdr.w, 2 * j + 1, s1, m1);
    return (d * (float)s0) * slo - (dmin * (float)m0) * xs_lo + (d * (float)s1) * shi -
           (dmin * (float)m1) * xs_hi;
}

// Q5_K unit: as Q4_K with the fifth bit from qh (bits 2j, 2j+1).
__device__ __forceinline__ float unit_q5k(const uint8_t *row, int u, const float *xr, float xs_lo,
                                          float xs_hi)
{
    const uint8_t *blk = row + (u >> 2) * 176;
    const int j = u & 3;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 ha = *reinterpret_cast<const uint4 *>(blk + 16);
    const uint4 hb = *reinterpret_cast<const uint4 *>(blk + 32);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * j);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    // Move bit 2j of every qh byte to bit 4 and bit 2j+1 to bit 4 of a
    // second word, so each lands where the fifth quant bit belongs.
    const uint32_t h[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    float slo = 0.0f, shi = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t hlo = ((h[k] >> (2 * j)) & 0x01010101u) << 4;
        const uint32_t hhi = ((h[k] >> (2 * j + 1)) & 0x01010101u) << 4;
        const uint32_t qlo = (w[k] & 0x0F0F0F0Fu) | hlo;
        const uint32_t qhi = ((w[k] >> 4) & 0x0F0F0F0Fu) | hhi;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            slo = fmaf(u2f_small((qlo >> (8 * b)) & 31u), xr[4 * k + b], slo);
            shi = fmaf(u2f_small((qhi >> (8 * b)) & 31u), xr[32 + 4 * k + b], shi);
        }
    }
    const float d = h2f(hdr.x & 0xFFFFu), dmin = h2f(hdr.x >> 16);
    uint32_t s0, m0, s1, m1;
    scale_min_w(hdr.y, hdr.z, hdr.w, 2 * j, s0, m0);
    scale_min_w(hdr.y, hdr.z, hdr.w, 2 * j + 1, s1, m1);
    return (d * (float)s0) * slo - (dmin * (float)m0) * xs_lo + (d * (float)s1) * shi -
           (dmin * (float)m1) * xs_hi;
}

// Q6_K unit: columns 128h + 64mm + [0, 64) of block u/4. Weight
// 128h + 64mm + 32k + l uses ql[64h + 32k + l] (low nibble if mm = 0, high
// if mm = 1) and bits 2(2mm + k) of qh[32h + l]; q - 32 times the int8 scale
// of its 16-weight group, times d.
__device__ __forceinline__ float unit_q6k(const uint8_t *row, int u, const float *xr)
{
    const uint8_t *blk = row + (u >> 2) * 210;
    const int h = (u >> 1) & 1, mm = u & 1;
    uint32_t ql[16], qh[8];
    ld_words_a2<16>(blk + 64 * h, ql);
    ld_words_a2<8>(blk + 128 + 32 * h, qh);
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int hs = 2 * (2 * mm + k);
#pragma unroll
        for (int wv = 0; wv < 8; wv++) {  // 8 words = 32 l values
            const uint32_t nib = mm ? ((ql[8 * k + wv] >> 4) & 0x0F0F0F0Fu) : (ql[8 * k + wv] & 0x0F0F0F0Fu);
            const uint32_t q6 = nib | (((qh[wv] >> hs) & 0x03030303u) << 4);
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int col = 32 * k + 4 * wv + b;  // within the unit
                // q - 32 exactly: (2^23 + q) - (2^23 + 32)
                const float qf = __uint_as_float(0x4B000000u | ((q6 >> (8 * b)) & 63u)) - 8388640.0f;
                s[col >> 4] = fmaf(qf, xr[col], s[col >> 4]);
            }
        }
    }
    const float d = h2f(ld_u16(blk + 208));
    const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * h + 4 * mm);
    return (d * (float)sc[0]) * s[0] + (d * (float)sc[1]) * s[1] + (d * (float)sc[2]) * s[2] +
           (d * (float)sc[3]) * s[3];
}

// Q4_0 unit: blocks 2u and (if present) 2u+1.
__device__ __forceinline__ float unit_q4_0(const uint8_t *row, int u, int nblocks, const float *xr)
{
    float total = 0.0f;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        if (2 * u + k < nblocks) {
            const uint8_t *blk = row + (2 * u + k) * 18;
            uint32_t w[4];
            ld_words_a2<4>(blk + 2, w);
            float s = 0.0f;
#pragma unroll
            for (int wv = 0; wv < 4; wv++) {
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    const uint32_t byte = (w[wv] >> (8 * b)) & 255u;
                    s = fmaf(__uint_as_float(0x4B000000u | (byte & 15u)) - 8388616.0f,
                             xr[32 * k + 4 * wv + b], s);
                    s = fmaf(__uint_as_float(0x4B000000u | (byte >> 4)) - 8388616.0f,
                             xr[32 * k + 16 + 4 * wv + b], s);
                }
            }
            total = fmaf(h2f(ld_u16(blk)), s, total);
        }
    }
    return total;
}

// Q8_0 unit: blocks 2u and (if present) 2u+1.
__device__ __forceinline__ float unit_q8_0(const uint8_t *row, int u, int nblocks, const float *xr)
{
    float total = 0.0f;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        if (2 * u + k < nblocks) {
            const uint8_t *blk = row + (2 * u + k) * 34;
            uint32_t w[8];
            ld_words_a2<8>(blk + 2, w);
            float s = 0.0f;
#pragma unroll
            for (int wv = 0; wv < 8; wv++) {
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    // signed byte -> (2^23 + 128 + q) - (2^23 + 128)
                    const uint32_t byte = ((w[wv] >> (8 * b)) & 255u) ^ 128u;
                    s = fmaf(__uint_as_float(0x4B000000u | byte) - 8388736.0f, xr[32 * k + 4 * wv + b], s);
                }
            }
            total = fmaf(h2f(ld_u16(blk)), s, total);
        }
    }
    return total;
}

// F32 / F16 unit: columns 64u .. min(64u+64, cols).
__device__ __forceinline__ float unit_float(int t, const uint8_t *row, int u, int cols, const float *xr)
{
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; i++) {
        const int c = 64 * u + i;
        if (c < cols) {
            s = fmaf(t == T_F32 ? decode_elem<T_F32>(row, c) : decode_elem<T_F16>(row, c), xr[i], s);
        }
    }
    return s;
}

}  // namespace pk
