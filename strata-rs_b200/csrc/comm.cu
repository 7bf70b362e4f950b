// comm.cu — multi-GPU state (NCCL) attached to a context.
#include "runtime.cuh"

namespace strata {

struct CommState {
    int rank = 0, world = 1;
};

void comm_release(strata_ctx* ctx) {
    delete ctx->comm;
    ctx->comm = nullptr;
}

}  // namespace strata
