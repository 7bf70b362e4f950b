// dequant.cu — bit-exact block dequantisation on the device.
//
// Each element is computed with the reference's own operation order and one
// rounding per operation (__fmul_rn / __fsub_rn / __fadd_rn cannot be fused
// into an FMA), so the output is bit-identical to strata-gguf's
// dequantize_row (crates/strata-gguf/src/dequant.rs:45-61).
//
// Non-finite scales: the reference runs on x86-64, whose SSE/AVX arithmetic
// returns the (quietened) NaN operand when one input is NaN, the first
// operand's when both are, and the negative "indefinite" NaN 0xFFC00000 for
// an invalid operation on non-NaN inputs (inf * 0, inf - inf). CUDA returns a
// canonical NaN instead, so each operation below re-derives the x86 result
// whenever its CUDA result is NaN.
#include "quant.cuh"
#include "kernels.cuh"

namespace strata {

__device__ __forceinline__ float x86_nan(float r, float a, float b) {
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xFFC00000u);
}
__device__ __forceinline__ float mul_x86(float a, float b) { return x86_nan(__fmul_rn(a, b), a, b); }
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
    } else {
        return 0.0f;
    }
}

template <uint32_t Q>
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ w, int64_t row_bytes, int64_t cols,
                                    int64_t nrows, float* __restrict__ out) {
    constexpr int BE = block_elems(Q), BB = block_bytes(Q);
    const int64_t total = nrows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / cols, c = i - r * cols;
        const uint8_t* blk = w + r * row_bytes + (c / BE) * BB;
        out[i] = dequant_elem<Q>(blk, (int)(c % BE));
    }
}

int launch_dequant(uint32_t quant, const uint8_t* w, int64_t row_bytes, int64_t cols, int64_t nrows,
                   float* out, cudaStream_t stream) {
    int64_t total = nrows * cols;
    if (total <= 0) return 0;
    int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 64) blocks = 148 * 64;
    switch (quant) {
#define STRATA_DQ(QID)                                                                              \
    case QID:                                                                                       \
        dequant_rows_kernel<QID><<<(unsigned)blocks, threads, 0, stream>>>(w, row_bytes, cols, nrows, out); \
        break;
        STRATA_DQ(kF32) STRATA_DQ(kF16) STRATA_DQ(kBF16) STRATA_DQ(kQ8_0)
        STRATA_DQ(kQ4_K) STRATA_DQ(kQ5_K) STRATA_DQ(kQ6_K)
#undef STRATA_DQ
    default:
        return -1;
    }
    return 0;
}

}  // namespace strata
