// dequant_elem.cuh — one element of a block, bit-exact against strata-gguf's
// dequantize_row (crates/strata-gguf/src/dequant.rs:45-61).
//
// Each element is computed with the reference's own operation order and one
// rounding per operation (__fmul_rn / __fsub_rn / __fadd_rn cannot be fused
// into an FMA), so the output is bit-identical to the reference.
//
// Non-finite scales: the reference runs on x86-64, whose SSE/AVX arithmetic
// returns the (quietened) NaN operand when one input is NaN, the first
// operand's when both are, and the negative "indefinite" NaN 0xFFC00000 for
// an invalid operation on non-NaN inputs (inf * 0, inf - inf). CUDA returns a
// canonical NaN instead, so each operation below re-derives the x86 result
// whenever its CUDA result is NaN.
//
// Layouts of the formats beyond the benchmark's four (bytes / elements):
//   Q4_0   18 / 32  [d][qs 16]: (nibble - 8) d, low nibbles j, high j + 16      (dequant.rs:138-144)
//   Q4_1   20 / 32  [d][m][qs 16]: nibble d + m                                  (dequant.rs:146-153)
//   Q5_0   22 / 32  [d][qh u32][qs 16]: 5th bit j / j + 16 of qh; (x - 16) d     (dequant.rs:155-166)
//   Q5_1   24 / 32  [d][m][qh u32][qs 16]: x d + m                               (dequant.rs:168-180)
//   Q8_1   36 / 32  [d][s][qs i8 x32]: q d                                       (dequant.rs:130-136)
//   Q2_0   18 / 64  [d][codes 16]: 2-bit codes LSB first, (code - 1) d           (dequant.rs:87-96)
//   IQ4_NL 18 / 32  [d][qs 16]: d codebook[nibble]                               (dequant.rs:182-189)
//   IQ4_XS 136/256  [d][scales_h u16][scales_l 4][qs 128]: 8 sub-blocks of 32,
//                   dl = d (ls - 32), ls 6 bits; every sub-block reads qs[0..16]
//                   (strata-gguf's loop does not advance qs)                   (dequant.rs:191-206)
//   Q2_K   84 /256  [d][dmin][scales 16][qs 64]: 2-bit fields, (s, m) of
//                   get_scale_min_k4                                            (dequant.rs:351-380)
//   Q3_K   110/256  [hmask 32][qs 64][scales 12][d @108]: 2-bit quants, -4
//                   unless the hmask bit is set, 16 6-bit scales - 32          (dequant.rs:304-349)
//   MXFP4  17 / 32  [e8m0][qs 16]: 2^(e-127) fp4 / 2 (E2M1 in half units)     (dequant.rs:382-424)
//   NVFP4  36 / 64  [ue4m3 x4][qs 32]: sub-block s of 16: value j in the low
//                   nibble of qs[8s + j], j + 8 in the high one                (dequant.rs:397-444)
#pragma once
#include "quant.cuh"

namespace strata {


__device__ __forceinline__ float x86_nan(float r, float a, float b) {
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xFFC00000u);
}
__device__ __forceinline__ float mul_x86(float a, float b) { return x86_nan(__fmul_rn(a, b), a, b); }

// The IQ4_NL codebook (the 16 values a 4-bit index selects; IQ4_NL and IQ4_XS,
// crates/strata-gguf/src/tables.rs KVALUES_IQ4NL): a format constant.
__device__ __forceinline__ int iq4nl_value(uint32_t i) {
    constexpr int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    return kv[i & 15];
}
// E2M1 (FP4) code in half units, from the format: magnitudes 0, 0.5, 1, 1.5,
// 2, 3, 4, 6 doubled; bit 3 the sign; code 8 is +0 (the table's 0).
__device__ __forceinline__ float fp4_half_units(uint32_t code) {
    const uint32_t e = (code >> 1) & 3u, mb = code & 1u;
    const uint32_t mag = e == 0 ? mb : (2u + mb) << (e - 1);
    return (code & 8u) && mag ? -(float)mag : (float)mag;
}
// UE4M3 scale (dequant.rs:397-413): no infinities, 0x7F / 0xFF NaN.
__device__ __forceinline__ float ue4m3_value(uint32_t e) {
    const int ex = (e >> 3) & 0xF, man = e & 7;
    float v;
    if (ex == 0) v = __fmul_rn(__fdiv_rn((float)man, 8.0f), 0.015625f);
    else if (ex == 15 && man == 7) v = __uint_as_float(0x7FC00000u);
    else v = __fmul_rn(__uint_as_float((uint32_t)(ex - 7 + 127) << 23), __fadd_rn(1.0f, __fdiv_rn((float)man, 8.0f)));
    return (e & 0x80u) ? -v : v;
}
__device__ __forceinline__ float sub_x86(float a, float b) { return x86_nan(__fsub_rn(a, b), a, b); }
__device__ __forceinline__ float add_x86(float a, float b) { return x86_nan(__fadd_rn(a, b), a, b); }

__device__ __forceinline__ uint32_t rd16(const uint8_t* b) { return (uint32_t)b[0] | ((uint32_t)b[1] << 8); }

// One output element `j` (0..block_elems-1) of the block at `b`.
template <uint32_t Q>
__device__ __forceinline__ float dequant_elem(const uint8_t* b, int j) {
    if constexpr (Q == kF32) {
        uint32_t u = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
        return __uint_as_float(u);
    } else if constexpr (Q == kF16) {
        return f16_bits_to_f32_exact(rd16(b));
    } else if constexpr (Q == kBF16) {
        return __uint_as_float(rd16(b) << 16);
    } else if constexpr (Q == kQ8_0) {
        // dequant.rs:123-128: (qs[j] as i8) as f32 * d
        float d = f16_bits_to_f32_exact(rd16(b));
        return mul_x86((float)(int8_t)b[2 + j], d);
    } else if constexpr (Q == kQ4_K) {
        // dequant.rs:247-270: chunk c of 64, low nibbles then high nibbles
        float d = f16_bits_to_f32_exact(rd16(b));
        float mn = f16_bits_to_f32_exact(rd16(b + 2));
        int c = j >> 6, l = j & 63, hi = l >> 5;
        uint32_t sc, m;
        scale_min_k4(2 * c + hi, b + 4, sc, m);
        uint32_t byte = b[16 + 32 * c + (l & 31)];
        uint32_t q = hi ? (byte >> 4) : (byte & 0xFu);
        float d1 = mul_x86(d, (float)sc), m1 = mul_x86(mn, (float)m);
        return sub_x86(mul_x86(d1, (float)q), m1);
    } else if constexpr (Q == kQ5_K) {
        // dequant.rs:272-302: + 16 when the qh bit (u1 / u2 = 1 << (2c + hi)) is set
        float d = f16_bits_to_f32_exact(rd16(b));
        float mn = f16_bits_to_f32_exact(rd16(b + 2));
        int c = j >> 6, l = j & 63, hi = l >> 5, ll = l & 31;
        uint32_t sc, m;
        scale_min_k4(2 * c + hi, b + 4, sc, m);
        uint32_t byte = b[48 + 32 * c + ll];
        uint32_t q = hi ? (byte >> 4) : (byte & 0xFu);
        float h = (b[16 + ll] & (1u << (2 * c + hi))) ? 16.0f : 0.0f;
        float d1 = mul_x86(d, (float)sc), m1 = mul_x86(mn, (float)m);
        return sub_x86(mul_x86(d1, add_x86((float)q, h)), m1);
    } else if constexpr (Q == kQ6_K) {
        // dequant.rs:208-234: halves of 128; quarter g = l / 32 selects
        // (ql lo / ql+32 lo / ql hi / ql+32 hi) and qh bits 2g..2g+1; u8 scales
        float d = f16_bits_to_f32_exact(rd16(b + 208));
        int half = j >> 7, r = j & 127, g = r >> 5, l = r & 31;
        const uint8_t* ql = b + 64 * half;
        const uint8_t* qh = b + 128 + 32 * half;
        const uint8_t* sc = b + 192 + 8 * half;
        uint32_t qlb = ql[l + ((g & 1) ? 32 : 0)];
        uint32_t nib = (g >= 2) ? (qlb >> 4) : (qlb & 0xFu);
        int q = (int)(nib | (((qh[l] >> (2 * g)) & 3u) << 4)) - 32;
        float s = (float)sc[(l >> 4) + 2 * g];
        return mul_x86(mul_x86(d, s), (float)q);
    } else if constexpr (Q == kQ4_0 || Q == kIQ4_NL) {
        const float d = f16_bits_to_f32_exact(rd16(b));
        const uint32_t byte = b[2 + (j & 15)];
        const uint32_t nib = j < 16 ? (byte & 0xFu) : (byte >> 4);
        if constexpr (Q == kQ4_0) return mul_x86(sub_x86((float)nib, 8.0f), d);
        else return mul_x86(d, (float)iq4nl_value(nib));
    } else if constexpr (Q == kQ4_1) {
        const float d = f16_bits_to_f32_exact(rd16(b)), m = f16_bits_to_f32_exact(rd16(b + 2));
        const uint32_t byte = b[4 + (j & 15)];
        return add_x86(mul_x86((float)(j < 16 ? (byte & 0xFu) : (byte >> 4)), d), m);
    } else if constexpr (Q == kQ5_0 || Q == kQ5_1) {
        constexpr int H = Q == kQ5_0 ? 2 : 4;  // qh offset; quants follow it
        const float d = f16_bits_to_f32_exact(rd16(b));
        const uint32_t h = (uint32_t)b[H] | ((uint32_t)b[H + 1] << 8) | ((uint32_t)b[H + 2] << 16) |
                           ((uint32_t)b[H + 3] << 24);
        const uint32_t byte = b[H + 4 + (j & 15)];
        const uint32_t x = (j < 16 ? (byte & 0xFu) : (byte >> 4)) | (((h >> j) & 1u) << 4);
        if constexpr (Q == kQ5_0) return mul_x86(sub_x86((float)x, 16.0f), d);
        else return add_x86(mul_x86((float)x, d), f16_bits_to_f32_exact(rd16(b + 2)));
    } else if constexpr (Q == kQ8_1) {
        return mul_x86((float)(int8_t)b[4 + j], f16_bits_to_f32_exact(rd16(b)));
    } else if constexpr (Q == kQ2_0) {
        const uint32_t code = (b[2 + (j >> 2)] >> ((j & 3) * 2)) & 3u;
        return mul_x86(sub_x86((float)code, 1.0f), f16_bits_to_f32_exact(rd16(b)));
    } else if constexpr (Q == kIQ4_XS) {
        const float d = f16_bits_to_f32_exact(rd16(b));
        const int ib = j >> 5, l = j & 31;
        const uint32_t ls = ((b[4 + (ib >> 1)] >> (4 * (ib & 1))) & 0xFu) | (((rd16(b + 2) >> (2 * ib)) & 3u) << 4);
        const float dl = mul_x86(d, sub_x86((float)ls, 32.0f));
        // every sub-block reads the first 16 quant bytes, as dequant.rs:194-203 does
        const uint32_t byte = b[8 + (l & 15)];
        return mul_x86(dl, (float)iq4nl_value(l < 16 ? (byte & 0xFu) : (byte >> 4)));
    } else if constexpr (Q == kQ2_K) {
        // 128-element groups g; within, 2-bit field f = (j % 128) / 32 of byte l, sub-block 2g + (f & 1)
        const float d = f16_bits_to_f32_exact(rd16(b)), mn = f16_bits_to_f32_exact(rd16(b + 2));
        const int g = j >> 7, f = (j & 127) >> 5, l = j & 31;
        uint32_t sc, m;
        scale_min_k4(2 * g + (f & 1), b + 4, sc, m);
        const uint32_t q = (b[20 + 32 * g + l] >> (2 * f)) & 3u;
        return sub_x86(mul_x86(mul_x86(d, (float)sc), (float)q), mul_x86(mn, (float)m));
    } else if constexpr (Q == kQ3_K) {
        // half h of 128; shift s4 of 4 (32 elements each, two scales of 16); hmask bit 4h + s4
        const float d = f16_bits_to_f32_exact(rd16(b + 108));
        const int h = j >> 7, s4 = (j & 127) >> 5, l = j & 31;
        const int is = 8 * h + 2 * s4 + (l >> 4);
        // 6-bit scale is: low 4 bits from the nibbles of bytes 0..7, high 2 from bytes 8..11
        const uint32_t lo = is < 8 ? (b[96 + is] & 0xFu) : (b[96 + is - 8] >> 4);
        const uint32_t hi = (b[104 + (is & 3)] >> (2 * (is >> 2))) & 3u;
        const int sc = (int)(lo | (hi << 4)) - 32;
        const float dl = mul_x86(d, (float)sc);
        const int q = (b[32 + 32 * h + l] >> (2 * s4)) & 3;
        const float off = (b[l] & (1u << (4 * h + s4))) ? 0.0f : 4.0f;
        return mul_x86(dl, sub_x86((float)q, off));
    } else if constexpr (Q == kMXFP4) {
        const uint32_t e = b[0];
        const float d = e == 0 ? 0.0f : (e == 0xFF ? __uint_as_float(0x7FC00000u) : __uint_as_float(e << 23));
        const uint32_t byte = b[1 + (j & 15)];
        return mul_x86(mul_x86(d, fp4_half_units(j < 16 ? (byte & 0xFu) : (byte >> 4))), 0.5f);
    } else if constexpr (Q == kNVFP4) {
        const int s = j >> 4, l = j & 15;
        const float ds = ue4m3_value(b[s]);
        const uint32_t byte = b[4 + 8 * s + (l & 7)];
        return mul_x86(mul_x86(ds, fp4_half_units(l < 8 ? (byte & 0xFu) : (byte >> 4))), 0.5f);
    } else {
        return 0.0f;
    }
}

}  // namespace strata
