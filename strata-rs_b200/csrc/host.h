// host.h — what the plain C++ sources (no CUDA headers) need from runtime.cu.
#pragma once
#include <nvtx3/nvToolsExt.h>

#include <cstdint>

#include "../../include/strata_cuda.h"

namespace strata {

// An NVTX range around one C-ABI call, named after the entry point, so Nsight
// timelines (and ncu --nvtx filters) show each call; with no tool attached the
// push and pop are no-ops.
struct CallRange {
    explicit CallRange(const char* name) { nvtxRangePushA(name); }
    ~CallRange() { nvtxRangePop(); }
    CallRange(const CallRange&) = delete;
    CallRange& operator=(const CallRange&) = delete;
};

// Records `msg` as the context's last error (under its lock) and returns `code`.
int report(strata_ctx* ctx, int code, const char* msg);
// True when the device path has kernels for this Strata ggml type id.
bool quant_on_device(uint32_t quant);

}  // namespace strata

#define STRATA_CALL_RANGE() ::strata::CallRange strata_call_range_(__func__)
