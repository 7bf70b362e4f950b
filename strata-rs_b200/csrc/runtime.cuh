// runtime.cuh — the host-side state behind the opaque handles of strata_cuda.h.
#pragma once
#include "staging.h"
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_set>

#include "../../include/strata_cuda.h"
#include "host.h"
#include "kernels.cuh"
#include "quant.cuh"

namespace strata {

struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
};
struct PinnedBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    void* dev = nullptr;  // the same memory's device address (unified addressing: usually ptr itself)
};

struct CommState;  // comm.cu

}  // namespace strata

struct strata_ctx {
    int device = 0;
    int sm_count = 0;
    int l2_bytes = 0;
    int cc_major = 0, cc_minor = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    std::mutex mu;
    std::string last_error;
    uint64_t budget_bytes = 0;
    uint64_t resident_bytes = 0;
    uint32_t wait_timeout_ms = 60000;
    int gemv_path = 0;  // STRATA_GEMV_AUTO / _CUDA_CORES / _TENSOR_CORES
    int gemm_terms = 2;  // bf16 terms per staged GEMM weight
    strata::DevBuf x_dev, y_dev, work, xfrag, gemm_work, x_bf16, moe_work;
    // the MoE layer's shared expert runs on `aux` (highest priority: decode,
    // where it races the routed chain for SM slots) or `aux_lo` (default
    // priority: many tokens, where the routed passes are the long pole),
    // forked from and joined back into the caller's stream (created with the
    // first MoE layer)
    cudaStream_t aux = nullptr, aux_lo = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    strata::PinnedBuf x_host, y_host;
    // host-buffer calls: the result comes back in pieces, each copied out to
    // the caller (by the pool's threads) while the next is still in transfer
    static constexpr int kPieces = 4;
    cudaEvent_t piece_ev[kPieces] = {};
    // a large GEMV result computed as row slices: slice k's rows leave on
    // `copy` (created with the first such call) once slice_ev[k] says they are done
    cudaStream_t copy = nullptr;
    cudaEvent_t slice_ev[kPieces] = {};
    strata::CopyPool copy_pool;
    // upload staging: two pinned chunks filled by host threads while the
    // other one is copied to the device (large tensors), with their events
    strata::PinnedBuf stage[2];
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
    // every weight uploaded and not yet freed (released by strata_cuda_destroy)
    std::unordered_set<strata_weight*> weights;
    // every MoE layer created and not yet destroyed: strata_cuda_destroy
    // releases their captured graphs and detaches them
    std::unordered_set<strata_moe*> moes;
    strata::CommState* comm = nullptr;
    int* err_host = nullptr;  // host-mapped word kernels set when a bounded wait expires
    int* err_dev = nullptr;
    // bumped whenever ensure_device / ensure_pinned (re)allocates a buffer
    // or the GEMV path changes: a captured graph that reads the context's
    // buffers is valid only for the generation it was captured in
    uint64_t buf_gen = 0;
};

constexpr uint32_t kWeightMagic = 0x57545253u;  // "SRTW"

struct strata_weight {
    uint32_t magic = kWeightMagic;
    strata_ctx* ctx = nullptr;
    uint32_t quant = 0;
    int64_t n_expert = 0, rows = 0, cols = 0, row_bytes = 0;
    uint8_t* dev = nullptr;
    size_t bytes = 0;
    alignas(64) unsigned char tmap[128];  // tensor map of a dense Q4_K / Q5_K matrix for the GEMV
    bool has_tmap = false;
};

namespace strata {

int fail(strata_ctx* ctx, int code, const char* fmt, ...);
int cuda_fail(strata_ctx* ctx, cudaError_t e, const char* what);
int64_t quant_row_bytes(uint32_t quant, int64_t cols);
int ensure_device(strata_ctx* ctx, DevBuf& b, size_t bytes, const char* what);
int ensure_pinned(strata_ctx* ctx, PinnedBuf& b, size_t bytes, const char* what);
int wait_stream(strata_ctx* ctx, cudaStream_t s);
cudaStream_t pick_stream(strata_ctx* ctx, void* stream);
int check_launch(strata_ctx* ctx, const char* what);
int check_weight(strata_ctx* ctx, const strata_weight* w, bool expert);

// expert.cu
int64_t expert_gemv_work_floats(int64_t IN, int64_t OUT, int sm_count);
int launch_expert_gemv_ws(uint32_t quant, const ExpertGemvArgs& a, float* work, int64_t work_floats,
                          cudaStream_t s);

// gemv_mma.cu (launchers declared in kernels.cuh)
bool encode_gemv_tmap(uint32_t quant, const void* base, int64_t rows, int64_t row_bytes, void* out128);
int check_device_error(strata_ctx* ctx);

// runtime.cu: enqueue on a stream (the context lock is held by the caller)
int gemv_enqueue(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                 cudaStream_t s);
int gemv_enqueue_strided(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                         int64_t ldy, cudaStream_t s, const PeerOut* peers = nullptr);
bool gemv_peer_capable(strata_ctx* ctx, const strata_weight* w, const float* x_dev, int batch);
int gemm_enqueue(strata_ctx* ctx, const strata_weight* w, const uint16_t* x_dev, float* y_dev, int64_t m,
                 cudaStream_t s);

// moe_host.cu
int moe_enqueue_checked(strata_ctx* ctx, const strata_moe* layer, const float* x, const float* logits, int64_t T,
                        float* out, int32_t* ids, float* wts, cudaStream_t s);
int64_t moe_embd(const strata_moe* layer);

// comm.cu
void comm_release(strata_ctx* ctx);

// moe_host.cu: the context's layers give up their graphs and their context
void moe_release_all(strata_ctx* ctx);

}  // namespace strata
