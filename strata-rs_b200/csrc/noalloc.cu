// noalloc.cu — the decode GEMV for callers that cannot allocate device memory.
//
// strata_cuda_gemv_noalloc runs the same tensor-core GEMV as strata_cuda_gemv_dev
// (activation-limb prologue + TMA-staged mma.sync kernel), but takes the weights
// as a plain device pointer, needs no context, and keeps its scratch (the
// activation limbs, their scales and per-sub-block sums) in the file-scope
// array below instead of a context workspace. Nothing here calls cudaMalloc,
// cudaFree or any allocating library routine.
#include <mutex>

#include "runtime.cuh"

namespace strata {
namespace {

// Scratch for one call: at most cols * batch = 65,536 (e.g. K = 8192 at batch 8,
// K = 65,536 at batch 1) needs about 266 KiB; 320 KiB are reserved. The array
// is part of the library's device image, so every GPU that loads the library
// holds it until the process exits.
constexpr size_t kNoallocScratchBytes = 320u << 10;
constexpr int64_t kNoallocMaxColsTimesBatch = 65536;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];
// Set by a kernel whose bounded wait on its shared-memory copies expired.
static __device__ int g_noalloc_err;

constexpr int kMaxDevices = 64;
struct DeviceSlot {
    bool ready = false;
    void* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int* err = nullptr;       // device address of g_noalloc_err on this device
    int sm_count = 0;
};
DeviceSlot g_slots[kMaxDevices];
std::mutex g_slots_mu;

// Once per device, with that device current: the device addresses of the
// static arrays (in host code their names are only host-side stand-ins).
int setup_device(int dev, DeviceSlot** out) {
    if (dev < 0 || dev >= kMaxDevices) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(g_slots_mu);
    DeviceSlot& s = g_slots[dev];
    if (!s.ready) {
        void* scratch = nullptr;
        void* err = nullptr;
        if (cudaGetSymbolAddress(&scratch, g_noalloc_scratch) != cudaSuccess || !scratch) return STRATA_ERR_CUDA;
        if (cudaGetSymbolAddress(&err, g_noalloc_err) != cudaSuccess || !err) return STRATA_ERR_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
            return STRATA_ERR_CUDA;
        s.scratch = scratch;
        s.err = reinterpret_cast<int*>(err);
        s.sm_count = sms;
        s.ready = true;
    }
    *out = &s;
    return STRATA_OK;
}

}  // namespace
}  // namespace strata

using namespace strata;

extern "C" int strata_cuda_gemv_noalloc(const uint8_t* w_dev, uint32_t quant, int64_t rows, int64_t cols,
                                        const float* x_dev, float* y_dev, int batch, void* stream) {
    if (quant != kQ4_K && quant != kQ5_K) return STRATA_ERR_UNSUPPORTED_QUANT;
    if (!w_dev || !x_dev || !y_dev || rows <= 0 || cols <= 0 || batch < 1 || batch > 8) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    if (cols % 256 != 0) return STRATA_ERR_TRUNCATED;
    if (cols * batch > kNoallocMaxColsTimesBatch) return STRATA_ERR_SCRATCH_LIMIT;
    if (((uintptr_t)w_dev & 15) || ((uintptr_t)x_dev & 15) || ((uintptr_t)y_dev & 3)) return STRATA_ERR_INVALID;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return STRATA_ERR_CUDA;
    DeviceSlot* slot = nullptr;
    int rc = setup_device(dev, &slot);
    if (rc) return rc;
    const int64_t row_bytes = quant_row_bytes(quant, cols);
    GemvArgs a{w_dev, row_bytes, rows, cols, x_dev, y_dev, batch, slot->sm_count, nullptr};
    if (!gemv_mma_supported(quant, a)) return STRATA_ERR_INVALID;
    if (gemv_mma_work_bytes(cols, batch) + 1024 > (int64_t)kNoallocScratchBytes) return STRATA_ERR_SCRATCH_LIMIT;
    // the tensor map is a 128-byte host struct filled in place (no allocation)
    alignas(64) unsigned char tmap[128];
    if (encode_gemv_tmap(quant, w_dev, rows, row_bytes, tmap)) a.tmap = tmap;
    // an error left by earlier work is not this call's: report it without launching
    if (cudaPeekAtLastError() != cudaSuccess) return STRATA_ERR_CUDA;
    launch_gemv_mma(quant, a, slot->scratch, slot->err, reinterpret_cast<cudaStream_t>(stream));
    return cudaGetLastError() == cudaSuccess ? STRATA_OK : STRATA_ERR_CUDA;
}

// The kernels of strata_cuda_gemv_noalloc set g_noalloc_err when one of their
// bounded waits expires (their output is then incomplete). This reads it after
// the work queued on `stream`, without allocating: a device-to-host copy of
// one word into a local, then a wait for the stream.
extern "C" int strata_cuda_gemv_noalloc_status(void* stream, int clear) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return STRATA_ERR_CUDA;
    DeviceSlot* slot = nullptr;
    int rc = setup_device(dev, &slot);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int word = 0;
    if (cudaMemcpyAsync(&word, slot->err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return STRATA_ERR_CUDA;
    if (clear && word) {
        static const int zero = 0;
        if (cudaMemcpyAsync(slot->err, &zero, sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            return STRATA_ERR_CUDA;
    }
    return word ? STRATA_ERR_TIMEOUT : STRATA_OK;
}
