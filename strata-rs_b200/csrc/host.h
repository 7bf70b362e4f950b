// host.h — what the plain C++ sources (no CUDA headers) need from runtime.cu.
#pragma once
#include <cstdint>

#include "../../include/strata_cuda.h"

namespace strata {

// Records `msg` as the context's last error (under its lock) and returns `code`.
int report(strata_ctx* ctx, int code, const char* msg);
// True when the device path has kernels for this Strata ggml type id.
bool quant_on_device(uint32_t quant);

}  // namespace strata
