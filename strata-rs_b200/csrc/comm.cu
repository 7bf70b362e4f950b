// comm.cu — multi-GPU paths: one process per GPU, one NCCL communicator per
// context (the reference is single-device; these are the sharded forms of
// its gemv and MoE layer).
//
//   row-sharded projection  each rank holds rows [rank N/G, (rank + 1) N/G)
//                           of W, runs the local GEMV / GEMM into its slice
//                           and an all-gather assembles y = [B | M][N];
//   expert-parallel MoE     each rank holds experts [r E/G, (r + 1) E/G),
//                           computes their weighted partial sums for all
//                           tokens (routing is replicated: it is cheap and
//                           deterministic) and an all-reduce adds them.
//
// The communicator is created non-blocking, so a rank that never joins makes
// init fail with STRATA_ERR_TIMEOUT after the context's wait timeout instead
// of blocking forever; every NCCL call is followed by a bounded poll of the
// communicator state.
//
// NCCL is opened with dlopen("libnccl.so.2") the first time a communicator is
// needed, not linked: a process that already loaded NCCL (PyTorch does) gets
// that same copy, and single-GPU use never loads NCCL at all.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <type_traits>

#include "runtime.cuh"

namespace strata {

struct Nccl {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char* (*GetErrorString)(ncclResult_t);
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char* e = dlerror();
            n.why = e ? e : "dlopen(libnccl.so.2) failed";
            return;
        }
        bool all = true;
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) {
                all = false;
                n.why = std::string("libnccl.so.2 lacks ") + name;
            }
        };
        sym(n.GetUniqueId, "ncclGetUniqueId");
        sym(n.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(n.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(n.CommDestroy, "ncclCommDestroy");
        sym(n.CommAbort, "ncclCommAbort");
        sym(n.AllGather, "ncclAllGather");
        sym(n.AllReduce, "ncclAllReduce");
        sym(n.GroupStart, "ncclGroupStart");
        sym(n.GroupEnd, "ncclGroupEnd");
        sym(n.GetErrorString, "ncclGetErrorString");
        n.ok = all;
    });
    return n;
}

struct CommState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    int group_depth = 0;  // > 0 inside strata_cuda_comm_group_start / end
    DevBuf send, recv;    // gather staging of the GEMM (m > 1)
};

void comm_release(strata_ctx* ctx) {
    if (!ctx->comm) return;
    if (ctx->comm->comm) {
        ncclResult_t st = ncclSuccess;
        nccl().CommGetAsyncError(ctx->comm->comm, &st);
        if (st == ncclSuccess) nccl().CommDestroy(ctx->comm->comm);
        else nccl().CommAbort(ctx->comm->comm);
    }
    for (DevBuf* b : {&ctx->comm->send, &ctx->comm->recv})
        if (b->ptr) cudaFree(b->ptr);
    delete ctx->comm;
    ctx->comm = nullptr;
}

namespace {

// Completes a non-blocking NCCL call: polls the communicator until it leaves
// ncclInProgress, at most the context's wait timeout.
int nccl_done(strata_ctx* ctx, ncclComm_t comm, ncclResult_t r, const char* what) {
    auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress) {
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if ((uint64_t)ms > ctx->wait_timeout_ms)
            return fail(ctx, STRATA_ERR_TIMEOUT, "%s did not complete within %u ms", what, ctx->wait_timeout_ms);
        std::this_thread::yield();
        if (nccl().CommGetAsyncError(comm, &r) != ncclSuccess) break;
    }
    if (r != ncclSuccess) return fail(ctx, STRATA_ERR_NCCL, "%s: %s", what, nccl().GetErrorString(r));
    return STRATA_OK;
}

int need_comm(strata_ctx* ctx) {
    if (!ctx->comm || !ctx->comm->comm)
        return fail(ctx, STRATA_ERR_INVALID, "no communicator: call strata_cuda_comm_init first");
    return STRATA_OK;
}

// y[b][g ns + j] = part[g][b][j]
__global__ void gather_transpose_kernel(const float* __restrict__ part, float* __restrict__ y, int G, int B,
                                        int64_t ns) {
    const int64_t n = (int64_t)G * B * ns;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % ns, r = i / ns;
        const int64_t b = r % B, g = r / B;
        y[b * G * ns + g * ns + j] = part[i];
    }
}

// The all-gather of every rank's rows of y = [B][G ns]: one in-place
// all-gather per output row b (rank r's slice of row b is contiguous at
// y[b][r ns]), issued as one NCCL group, so no staging and no transpose. The
// local GEMV has already written this rank's slices in place.
int gather_rows_inplace(strata_ctx* ctx, float* y, int B, int64_t ns, cudaStream_t s) {
    CommState* c = ctx->comm;
    const int64_t N = ns * c->world;
    const bool own_group = c->group_depth == 0;
    int rc;
    if (own_group && (rc = nccl_done(ctx, c->comm, nccl().GroupStart(), "ncclGroupStart"))) return rc;
    for (int b = 0; b < B; ++b) {
        float* row = y + (int64_t)b * N;
        rc = nccl_done(ctx, c->comm, nccl().AllGather(row + c->rank * ns, row, (size_t)ns, ncclFloat, c->comm, s),
                       "ncclAllGather");
        if (rc) {
            if (own_group) nccl().GroupEnd();
            return rc;
        }
    }
    if (own_group) return nccl_done(ctx, c->comm, nccl().GroupEnd(), "ncclGroupEnd");
    return STRATA_OK;
}

// GEMM: [M][ns] per rank gathered into [G][M][ns], then transposed into [M][N].
int gather_rows_staged(strata_ctx* ctx, const float* local, float* y, int B, int64_t ns, cudaStream_t s) {
    CommState* c = ctx->comm;
    const int G = c->world;
    if (c->group_depth > 0)
        return fail(ctx, STRATA_ERR_INVALID, "the sharded GEMM cannot run inside a collective group");
    const size_t part = (size_t)B * (size_t)ns * 4;
    int rc = ensure_device(ctx, c->recv, part * (size_t)G, "cudaMalloc(gather)");
    if (rc) return rc;
    rc = nccl_done(ctx, c->comm, nccl().AllGather(local, c->recv.ptr, (size_t)B * (size_t)ns, ncclFloat, c->comm, s),
                   "ncclAllGather");
    if (rc) return rc;
    const int64_t n = (int64_t)G * B * ns;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 8 * (int64_t)ctx->sm_count) blocks = 8 * (int64_t)ctx->sm_count;
    gather_transpose_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, s>>>((const float*)c->recv.ptr, y, G, B,
                                                                                ns);
    return check_launch(ctx, "gather transpose kernel");
}

}  // namespace
}  // namespace strata

using namespace strata;

extern "C" {

int strata_cuda_comm_unique_id(uint8_t* id_out) {
    if (!id_out) return STRATA_ERR_INVALID;
    static_assert(sizeof(ncclUniqueId) == STRATA_COMM_ID_BYTES, "NCCL unique id size");
    if (!nccl().ok) return STRATA_ERR_NCCL;
    ncclUniqueId id;
    if (nccl().GetUniqueId(&id) != ncclSuccess) return STRATA_ERR_NCCL;
    memcpy(id_out, &id, sizeof(id));
    return STRATA_OK;
}

int strata_cuda_comm_init(strata_ctx* ctx, int rank, int world, const uint8_t* id_in) {
    if (!ctx || !id_in || world < 1 || rank < 0 || rank >= world) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    if (ctx->comm) return fail(ctx, STRATA_ERR_INVALID, "communicator already initialised");
    if (!nccl().ok) return fail(ctx, STRATA_ERR_NCCL, "NCCL unavailable: %s", nccl().why.c_str());
    cudaSetDevice(ctx->device);
    ncclUniqueId id;
    memcpy(&id, id_in, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    CommState* c = new CommState();
    c->rank = rank;
    c->world = world;
    ncclResult_t r = nccl().CommInitRankConfig(&c->comm, world, id, rank, &cfg);
    int rc = nccl_done(ctx, c->comm, r, "ncclCommInitRankConfig");
    if (rc) {
        if (c->comm) nccl().CommAbort(c->comm);
        delete c;
        return rc;
    }
    ctx->comm = c;
    return STRATA_OK;
}

int strata_cuda_comm_info(const strata_ctx* ctx, int* rank, int* world) {
    if (!ctx || !rank || !world) return STRATA_ERR_INVALID;
    *rank = ctx->comm ? ctx->comm->rank : 0;
    *world = ctx->comm ? ctx->comm->world : 1;
    return STRATA_OK;
}

int strata_cuda_comm_group_start(strata_ctx* ctx) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = need_comm(ctx);
    if (rc) return rc;
    if (ctx->comm->group_depth++ == 0)
        return nccl_done(ctx, ctx->comm->comm, nccl().GroupStart(), "ncclGroupStart");
    return STRATA_OK;
}

int strata_cuda_comm_group_end(strata_ctx* ctx) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = need_comm(ctx);
    if (rc) return rc;
    if (ctx->comm->group_depth == 0) return fail(ctx, STRATA_ERR_INVALID, "no collective group is open");
    if (--ctx->comm->group_depth == 0) return nccl_done(ctx, ctx->comm->comm, nccl().GroupEnd(), "ncclGroupEnd");
    return STRATA_OK;
}

int strata_cuda_gemv_sharded_dev(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                                 void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, false);
    if (rc || (rc = need_comm(ctx))) return rc;
    if (!x_dev || !y_dev) return fail(ctx, STRATA_ERR_INVALID, "null x or y");
    if (batch < 1 || batch > 8) return fail(ctx, STRATA_ERR_INVALID, "batch %d outside 1..8", batch);
    cudaSetDevice(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    CommState* c = ctx->comm;
    const int64_t ns = w->rows;
    // the local GEMV writes rank r's columns of every output row in place
    // (output row pitch N = world * ns)
    if ((rc = gemv_enqueue_strided(ctx, w, x_dev, y_dev + c->rank * ns, batch, ns * c->world, s))) return rc;
    return gather_rows_inplace(ctx, y_dev, batch, ns, s);
}

int strata_cuda_gemm_sharded_dev(strata_ctx* ctx, const strata_weight* w, const uint16_t* x_dev, float* y_dev,
                                 int64_t m, void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, false);
    if (rc || (rc = need_comm(ctx))) return rc;
    if (!x_dev || !y_dev) return fail(ctx, STRATA_ERR_INVALID, "null x or y");
    if (m < 1 || m >= (1 << 30)) return fail(ctx, STRATA_ERR_INVALID, "m %lld", (long long)m);
    cudaSetDevice(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    CommState* c = ctx->comm;
    const int64_t ns = w->rows;
    float* local = y_dev + c->rank * ns;
    if (m > 1) {
        if ((rc = ensure_device(ctx, c->send, (size_t)m * (size_t)ns * 4, "cudaMalloc(shard)"))) return rc;
        local = (float*)c->send.ptr;
    }
    if ((rc = gemm_enqueue(ctx, w, x_dev, local, m, s))) return rc;
    if (m == 1) return gather_rows_inplace(ctx, y_dev, 1, ns, s);
    return gather_rows_staged(ctx, local, y_dev, (int)m, ns, s);
}

int strata_cuda_moe_ffn_ep_dev(strata_ctx* ctx, const strata_moe* layer, const float* x_dev,
                               const float* logits_dev, int64_t tokens, float* out_dev, void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = need_comm(ctx);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    if ((rc = moe_enqueue_checked(ctx, layer, x_dev, logits_dev, tokens, out_dev, nullptr, nullptr, s))) return rc;
    const int64_t n = tokens * moe_embd(layer);
    return nccl_done(ctx, ctx->comm->comm,
                     nccl().AllReduce(out_dev, out_dev, (size_t)n, ncclFloat, ncclSum, ctx->comm->comm, s),
                     "ncclAllReduce");
}

}  // extern "C"
