// kernels.cuh — launchers shared between the kernel files and the runtime.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace strata {

// Dense GEMV arguments: W is N rows of `row_bytes` (rows = OUT, quantized
// along K = IN); X is batch x K f32, Y is batch x N f32, both row-major.
struct GemvArgs {
    const uint8_t* W;
    int64_t row_bytes;
    int64_t N, K;
    const float* X;
    float* Y;
    int batch;
    int sm_count;
    const void* tmap = nullptr;  // CUtensorMap of W for the tensor-core GEMV, or null
};

int launch_dequant(uint32_t quant, const uint8_t* w, int64_t row_bytes, int64_t cols, int64_t nrows,
                   float* out, cudaStream_t stream);
int launch_gemv(uint32_t quant, const GemvArgs& a, cudaStream_t s);

// Expert GEMV on the transposed expert layout [E][IN rows][OUT cols]
// (rows quantized along OUT): Y[b][c] = sum_i X[b][i] * W_e[i][c].
struct ExpertGemvArgs {
    const uint8_t* W;     // base of expert e's [IN][OUT] matrix
    int64_t row_bytes;    // bytes of one IN row (OUT elements)
    int64_t IN, OUT;
    const float* X;       // batch x IN
    float* Y;             // batch x OUT
    int batch;
    int sm_count;
};

}  // namespace strata
