// dequant.cu — bit-exact block dequantisation on the device.
//
// Per element with dequant_elem (dequant_elem.cuh): bit-identical to
// strata-gguf's dequantize_row (crates/strata-gguf/src/dequant.rs:45-61).
#include "dequant_elem.cuh"
#include "kernels.cuh"

namespace strata {

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
        STRATA_DQ(kQ4_0) STRATA_DQ(kQ4_1) STRATA_DQ(kQ5_0) STRATA_DQ(kQ5_1) STRATA_DQ(kQ8_1)
        STRATA_DQ(kQ2_K) STRATA_DQ(kQ3_K) STRATA_DQ(kIQ4_NL) STRATA_DQ(kIQ4_XS) STRATA_DQ(kMXFP4)
        STRATA_DQ(kNVFP4) STRATA_DQ(kQ2_0)
#undef STRATA_DQ
    default:
        return -1;
    }
    return 0;
}

}  // namespace strata
