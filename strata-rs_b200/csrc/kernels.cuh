// kernels.cuh — launchers shared between the kernel files and the runtime.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace strata {

// Row-sharded GEMV whose all-gather runs over peer memory: the outputs go to
// this rank's exchange buffer instead of Y (half `epoch & 1`, layout
// [batch][ldy], this call's first value at float `off` of the half), where
// the all-gather kernel pushes them to the other ranks.
constexpr int kMaxPeers = 8;
struct PeerOut {
    float* y;                   // this rank's exchange buffer (both halves)
    const unsigned int* epoch;  // this rank's call counter (its parity picks the half)
    int64_t half_floats;        // floats per half of an exchange buffer
    int64_t off;                // float offset in a half of this launch's y[0][0]
    int G;                      // 0: no exchange (plain GEMV)
};

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
    int64_t ldy = 0;             // output row pitch in floats (0: N)
    const PeerOut* peers = nullptr;  // outputs to the peer exchange buffer (tensor-core GEMV only), or null
};
inline int64_t ldy_of(const GemvArgs& a) { return a.ldy > 0 ? a.ldy : a.N; }

int launch_dequant(uint32_t quant, const uint8_t* w, int64_t row_bytes, int64_t cols, int64_t nrows,
                   float* out, cudaStream_t stream);
// CUDA-core GEMV: every quant type, any batch (8-token chunks beyond 8)
int launch_gemv(uint32_t quant, const GemvArgs& a, cudaStream_t s);
// Q8_0 at batch 1-2 with K a multiple of 1024: rows staged by bulk copies
// (gemv_mma.cu); the same arithmetic, in the same order, as launch_gemv's
bool gemv_q8_0_bulk_supported(const GemvArgs& a);
void launch_gemv_q8_0_bulk(const GemvArgs& a, int* err, cudaStream_t s);

// Tensor-core GEMV (Q4_K / Q5_K): activation-limb prologue + GEMV kernel,
// any batch (8-token chunks beyond 8); `work` holds gemv_mma_work_bytes.
int64_t gemv_mma_work_bytes(int64_t K, int batch);
bool gemv_mma_supported(uint32_t quant, const GemvArgs& a);
int launch_gemv_mma(uint32_t quant, const GemvArgs& a, void* work, int* err, cudaStream_t s, bool prep = true);

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

// Prefill GEMM: Y[m][n] = sum_k X[m][k] * W[n][k]; X is M x K bf16 bits,
// Y is M x N f32, both row-major; W is N rows of `row_bytes` (Q4_K/Q5_K/Q6_K).
struct GemmArgs {
    const uint8_t* W;
    int64_t row_bytes;
    int64_t N, K;
    const uint16_t* X;
    float* Y;
    int64_t M;
    int terms;       // 2: weights staged as bf16 hi + lo (the parity path); 1: hi only
    int sm_count;
    int* err;        // set to 1 by a kernel whose bounded wait expired
    float* work;     // split-K partials, gemm_tc_work_floats() floats (null when that is 0)
};

bool gemm_tc_supported(uint32_t quant, const GemmArgs& a);
int gemm_tc_splits(const GemmArgs& a);
int64_t gemm_tc_work_floats(const GemmArgs& a);
int launch_gemm_tc(uint32_t quant, const GemmArgs& a, cudaStream_t s);
void launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, int sm_count, cudaStream_t s);

}  // namespace strata
