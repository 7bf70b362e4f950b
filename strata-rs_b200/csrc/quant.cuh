// quant.cuh — ggml block layouts as strata-gguf stores them, and the device
// helpers that decode them.
//
// Layouts (bytes), from crates/strata-gguf/src/dequant.rs and quant.rs:138-165
// (the other formats' in dequant_elem.cuh):
//   Q8_0  34 B / 32 elems : [d f16][qs i8 x32]                              (dequant.rs:123-128)
//   Q4_K 144 B / 256      : [d f16][dmin f16][scales 12][qs 128]            (dequant.rs:247-270)
//   Q5_K 176 B / 256      : [d f16][dmin f16][scales 12][qh 32][qs 128]     (dequant.rs:272-302)
//   Q6_K 210 B / 256      : [ql 128][qh 64][scales u8 x16][d f16 @208]      (dequant.rs:208-234)
// Weights are uploaded byte-for-byte, so these offsets are the HBM layout too.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace strata {

// Strata ggml type ids (crates/strata-gguf/src/quant.rs:15-43).
enum QuantId : uint32_t {
    kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_1 = 3, kQ5_0 = 6, kQ5_1 = 7, kQ8_0 = 8, kQ8_1 = 9, kQ2_K = 10,
    kQ3_K = 11, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14, kIQ4_NL = 20, kIQ4_XS = 23, kBF16 = 30, kMXFP4 = 39,
    kNVFP4 = 40, kQ2_0 = 42,
};

// QuantType::block_size / type_size (quant.rs:124-163) of the types this
// library runs; 0 for the others (upload rejects them).
__host__ __device__ constexpr int block_elems(uint32_t q) {
    return (q == kF32 || q == kF16 || q == kBF16) ? 1
         : (q == kQ4_0 || q == kQ4_1 || q == kQ5_0 || q == kQ5_1 || q == kQ8_0 || q == kQ8_1 || q == kIQ4_NL ||
            q == kMXFP4) ? 32
         : (q == kNVFP4 || q == kQ2_0) ? 64
         : (q == kQ2_K || q == kQ3_K || q == kQ4_K || q == kQ5_K || q == kQ6_K || q == kIQ4_XS) ? 256 : 0;
}
__host__ __device__ constexpr int block_bytes(uint32_t q) {
    return q == kF32 ? 4 : (q == kF16 || q == kBF16) ? 2
         : (q == kQ4_0 || q == kIQ4_NL || q == kQ2_0) ? 18 : q == kQ4_1 ? 20 : q == kQ5_0 ? 22 : q == kQ5_1 ? 24
         : q == kQ8_0 ? 34 : q == kQ8_1 ? 36 : q == kQ2_K ? 84 : q == kQ3_K ? 110 : q == kQ4_K ? 144
         : q == kQ5_K ? 176 : q == kQ6_K ? 210 : q == kIQ4_XS ? 136 : q == kMXFP4 ? 17 : q == kNVFP4 ? 36 : 0;
}
// The formats beyond the benchmark's (dequant, the generic GEMV and expert
// GEMV paths; no fused fast path).
__host__ __device__ constexpr bool is_other_format(uint32_t q) {
    return q == kQ4_0 || q == kQ4_1 || q == kQ5_0 || q == kQ5_1 || q == kQ8_1 || q == kQ2_K || q == kQ3_K ||
           q == kIQ4_NL || q == kIQ4_XS || q == kMXFP4 || q == kNVFP4 || q == kQ2_0;
}

// binary16 -> binary32 by integer ops, exact for every input. A NaN keeps its
// payload with the quiet bit set (the `half` crate's result), so the
// bit-exact dequant path matches the reference even on non-finite scales.
__device__ __forceinline__ float f16_bits_to_f32_exact(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1Fu) {
        bits = sign | (man ? (0x7FC00000u | (man << 13)) : 0x7F800000u);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            // subnormal: shift the leading one up to bit 10
            int lz = __clz(man) - 21;          // man < 2^10, so lz >= 1
            man = (man << lz) & 0x3FFu;
            bits = sign | ((uint32_t)(113 - lz) << 23) | (man << 13);
        }
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    return __uint_as_float(bits);
}

// Hardware conversion for the fused kernels (exact for finite values).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    return __half2float(__ushort_as_half((unsigned short)h));
}

// get_scale_min_k4 (dequant.rs:237-245): 6-bit scale and min of sub-block j.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, uint32_t& sc, uint32_t& m) {
    if (j < 4) {
        sc = q[j] & 63u;
        m = q[j + 4] & 63u;
    } else {
        sc = (q[j + 4] & 0x0Fu) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// All eight 6-bit scales (or mins) of a Q4_K/Q5_K block as bytes, from the
// three little-endian words of the 12-byte scale field:
//   sc[0..3] = s0 & 63            m[0..3] = s1 & 63
//   sc[4..7] = (s2 & 15) | (s0 >> 6) << 4
//   m[4..7]  = (s2 >> 4) | (s1 >> 6) << 4
// which is get_scale_min_k4 evaluated for j = 0..7 at once.
__device__ __forceinline__ void scales_k4_packed(uint32_t s0, uint32_t s1, uint32_t s2,
                                                 uint32_t& sc_lo, uint32_t& sc_hi,
                                                 uint32_t& m_lo, uint32_t& m_hi) {
    sc_lo = s0 & 0x3F3F3F3Fu;
    m_lo = s1 & 0x3F3F3F3Fu;
    sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
}

// Bounded spin for every wait on device memory written by someone else.
constexpr long long kSpinLimit = 1ll << 26;

}  // namespace strata
