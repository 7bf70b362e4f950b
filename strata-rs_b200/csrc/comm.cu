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
#include <vector>

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

// Exchange buffer of the peer all-gather, one per rank, opened by every
// other rank through CUDA IPC: control words, then two halves of
// kPeerHalfFloats floats. The sharded GEMVs write their columns into this
// rank's half; the all-gather kernel pushes them into the same place of every
// other rank's half and then copies the whole rows out. Consecutive gathers
// alternate halves and count arrivals per half: a peer one gather ahead
// writes and signals the other half, and none can be two ahead (its next
// gather needs this rank's signal).
struct PeerCtl {
    unsigned long long arrivals[2];  // peers' "pushed" signals received for half h
    unsigned long long expected[2];  // signals the gathers on half h so far have waited for
    unsigned int epoch;              // gathers so far (its parity picks the half)
    unsigned int pushed;             // CTAs of the running gather kernel done pushing
    unsigned int finished;           // CTAs of the running gather kernel done copying
    int barrier;                     // all-reduce operand of the teardown barrier
};
constexpr int64_t kPeerCtlBytes = 256;
constexpr int64_t kPeerHalfFloats = int64_t(8) << 20;  // 32 MiB per half

constexpr int kPeerSegs = 32;
// The outputs one all-gather kernel assembles: those of up to kPeerSegs
// sharded GEMVs (one call, or the calls of a collective group). Segment s is
// y[s] = [rows][G ns], at float off[s] of the half in every rank's buffer;
// rank q wrote columns [q ns, (q + 1) ns) of every row into its own buffer.
struct PeerSegs {
    float* y[kPeerSegs];
    int64_t off[kPeerSegs];  // a multiple of 4
    int rows[kPeerSegs];
    int ns4[kPeerSegs];      // columns per rank / 4
    char* base[kMaxPeers];   // every rank's exchange buffer as mapped here
    int rank, G, count;
};
// Sharded GEMVs issued since the last all-gather kernel.
struct PeerPending {
    PeerSegs segs{};
    int64_t floats = 0;  // of the half in use
    cudaStream_t stream = nullptr;
};

struct CommState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    int group_depth = 0;  // > 0 inside strata_cuda_comm_group_start / end
    DevBuf send, recv;    // gather staging of the GEMM (m > 1)
    // fused peer gather
    int gather_mode = STRATA_GATHER_AUTO;
    bool peer_ok = false;                // every rank mapped every exchange buffer
    char* xbuf = nullptr;                // this rank's exchange buffer
    char* peer_base[kMaxPeers] = {};     // every rank's exchange buffer as mapped here
    PeerPending pending;                 // inside a collective group
    // peer collectives (and the GEMVs that write the exchange buffer) run in
    // issue order on the device: a call on another stream than the previous
    // one waits for it through `order`
    cudaStream_t peer_stream = nullptr;
    cudaEvent_t order = nullptr;
};

namespace {
int nccl_done(strata_ctx* ctx, ncclComm_t comm, ncclResult_t r, const char* what);

__host__ __device__ PeerCtl* ctl_of(char* base) { return reinterpret_cast<PeerCtl*>(base); }
__host__ __device__ float* data_of(char* base) { return reinterpret_cast<float*>(base + kPeerCtlBytes); }

// Unmaps the peers' exchange buffers and frees this rank's. With `barrier`,
// first waits (bounded) until every rank has reached this point, so no rank
// frees a buffer that another is still writing to.
void peer_release(strata_ctx* ctx, bool barrier) {
    CommState* c = ctx->comm;
    if (!c->xbuf) return;
    if (barrier && c->peer_ok) {
        int* b = &ctl_of(c->xbuf)->barrier;
        if (nccl_done(ctx, c->comm, nccl().AllReduce(b, b, 1, ncclInt32, ncclSum, c->comm, ctx->stream),
                      "ncclAllReduce(barrier)") == STRATA_OK)
            wait_stream(ctx, ctx->stream);
    }
    for (int q = 0; q < c->world && q < kMaxPeers; ++q)
        if (q != c->rank && c->peer_base[q]) cudaIpcCloseMemHandle(c->peer_base[q]);
    cudaFree(c->xbuf);
    c->xbuf = nullptr;
    if (c->order) cudaEventDestroy(c->order);
    c->order = nullptr;
    c->peer_stream = nullptr;
    c->peer_ok = false;
    for (auto& p : c->peer_base) p = nullptr;
}
}  // namespace

void comm_release(strata_ctx* ctx) {
    if (!ctx->comm) return;
    if (ctx->comm->comm) {
        ncclResult_t st = ncclSuccess;
        nccl().CommGetAsyncError(ctx->comm->comm, &st);
        peer_release(ctx, st == ncclSuccess);
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

// What each rank publishes about its exchange buffer.
struct PeerRecord {
    cudaIpcMemHandle_t handle;
    char bus_id[32];
    int sm_count;
    int ok;
};

// Allocates this rank's exchange buffer and maps every other rank's (CUDA
// IPC handles exchanged with an NCCL all-gather). Collective: every rank runs
// the same NCCL calls whatever fails locally, and an all-reduce (min) of the
// ranks' outcomes decides, so all ranks agree on whether the peer gather is
// available. Peer mapping needs distinct GPUs of the same model (the arrival
// count of a call is computed locally from the launch shape).
int peer_setup(strata_ctx* ctx) {
    CommState* c = ctx->comm;
    const int G = c->world;
    PeerRecord mine{};
    mine.sm_count = ctx->sm_count;
    bool ok = G <= kMaxPeers;
    if (ok) {
        const size_t bytes = (size_t)kPeerCtlBytes + 2 * (size_t)kPeerHalfFloats * 4;
        ok = cudaMalloc((void**)&c->xbuf, bytes) == cudaSuccess;
        if (!ok) c->xbuf = nullptr;
        ok = ok && cudaMemsetAsync(c->xbuf, 0, kPeerCtlBytes, ctx->stream) == cudaSuccess;
        ok = ok && cudaIpcGetMemHandle(&mine.handle, c->xbuf) == cudaSuccess;
        ok = ok && cudaDeviceGetPCIBusId(mine.bus_id, sizeof(mine.bus_id), ctx->device) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&c->order, cudaEventDisableTiming) == cudaSuccess;
    }
    cudaGetLastError();
    mine.ok = ok;
    // exchange the records (device staging for NCCL)
    PeerRecord* rec_dev = nullptr;
    std::vector<PeerRecord> recs(G);
    if (cudaMalloc((void**)&rec_dev, sizeof(PeerRecord) * (G + 1)) != cudaSuccess)
        return cuda_fail(ctx, cudaGetLastError(), "cudaMalloc(peer records)");
    int* ok_dev = reinterpret_cast<int*>(rec_dev + G);
    int rc = STRATA_OK;
    if (cudaMemcpyAsync(rec_dev + c->rank, &mine, sizeof(mine), cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
        rc = cuda_fail(ctx, cudaGetLastError(), "cudaMemcpyAsync(peer record)");
    if (!rc)
        rc = nccl_done(ctx, c->comm,
                       nccl().AllGather(rec_dev + c->rank, rec_dev, sizeof(PeerRecord), ncclUint8, c->comm,
                                        ctx->stream),
                       "ncclAllGather(peer records)");
    if (!rc && cudaMemcpyAsync(recs.data(), rec_dev, sizeof(PeerRecord) * G, cudaMemcpyDeviceToHost, ctx->stream) !=
                   cudaSuccess)
        rc = cuda_fail(ctx, cudaGetLastError(), "cudaMemcpyAsync(peer records)");
    if (!rc) rc = wait_stream(ctx, ctx->stream);
    if (!rc) {
        for (int q = 0; q < G && ok; ++q) {
            ok = recs[q].ok && recs[q].sm_count == ctx->sm_count;
            for (int p = 0; p < q && ok; ++p) ok = strncmp(recs[p].bus_id, recs[q].bus_id, sizeof(recs[q].bus_id)) != 0;
        }
        for (int q = 0; q < G && ok; ++q) {
            if (q == c->rank) {
                c->peer_base[q] = c->xbuf;
                continue;
            }
            void* p = nullptr;
            ok = cudaIpcOpenMemHandle(&p, recs[q].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            c->peer_base[q] = ok ? static_cast<char*>(p) : nullptr;
        }
        cudaGetLastError();
        const int flag = ok ? 1 : 0;
        if (cudaMemcpyAsync(ok_dev, &flag, sizeof(int), cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
            rc = cuda_fail(ctx, cudaGetLastError(), "cudaMemcpyAsync(peer flag)");
        if (!rc)
            rc = nccl_done(ctx, c->comm, nccl().AllReduce(ok_dev, ok_dev, 1, ncclInt32, ncclMin, c->comm, ctx->stream),
                           "ncclAllReduce(peer flag)");
        int all = 0;
        if (!rc && cudaMemcpyAsync(&all, ok_dev, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
            rc = cuda_fail(ctx, cudaGetLastError(), "cudaMemcpyAsync(peer flag)");
        if (!rc) rc = wait_stream(ctx, ctx->stream);
        c->peer_ok = !rc && all == 1;
    }
    cudaFree(rec_dev);
    if (!c->peer_ok) peer_release(ctx, false);
    return rc;
}

// Bounded spin (thread 0) until *ctr >= target; false after timeout_ns.
__device__ bool wait_count(unsigned long long* ctr, unsigned long long target, uint64_t timeout_ns) {
    uint64_t t0, now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (long long i = 0; i < (1ll << 40); ++i) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (now - t0 > timeout_ns) return false;
        __nanosleep(64);
    }
    return false;
}

// The synchronisation every peer collective shares, run by all threads of
// every CTA of a cooperative launch (all CTAs resident: a CTA waits on
// signals that other ranks send only after all of this rank's CTAs arrived):
// every CTA releases its stores (system scope) and counts itself; the last
// one adds 1 to every other rank's arrival counter of half h; then each CTA
// waits (bounded) for the G - 1 other ranks' signals on half h. False (and
// *err set) if the wait expired.
__device__ bool peer_signal_wait(PeerCtl* ctl, char* const* base, int me, int G, unsigned int h, uint64_t timeout_ns,
                                 int* err) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        if (atomicAdd(&ctl->pushed, 1u) == gridDim.x - 1) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (int q = 0; q < G; ++q)
                if (q != me) atomicAdd_system(&ctl_of(base[q])->arrivals[h], 1ull);
        }
        const bool ok = wait_count(&ctl->arrivals[h], ctl->expected[h] + (unsigned long long)(G - 1), timeout_ns);
        if (!ok) atomicExch(err, 1);
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// The last CTA to finish advances half h's expected count and the epoch
// (every CTA has read both by then) and resets the CTA counters. After an
// expired wait the counts no longer match: the communicator has to be
// recreated before the next peer collective.
__device__ void peer_advance(PeerCtl* ctl, unsigned int e, int G) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&ctl->finished, 1u) == gridDim.x - 1) {
            ctl->expected[e & 1u] += (unsigned long long)(G - 1);
            ctl->epoch = e + 1;
            ctl->pushed = 0;
            ctl->finished = 0;
            __threadfence();
        }
    }
}

__device__ unsigned int peer_epoch(PeerCtl* ctl) {
    __shared__ unsigned int epoch_s;
    if (threadIdx.x == 0) epoch_s = *(volatile unsigned int*)&ctl->epoch;
    __syncthreads();
    return epoch_s;
}

// The all-gather of the pending segments, one cooperative launch:
//   1. push: this rank's columns of every row go from its own half to the
//      same place in every other rank's half (16-byte stores over NVLink) and
//      to y;
//   2. signal and wait (peer_signal_wait);
//   3. copy the other ranks' columns from this rank's half to y;
//   4. advance the epoch.
__global__ void peer_allgather_kernel(const __grid_constant__ PeerSegs segs, uint64_t timeout_ns, int* err) {
    char* own = segs.base[segs.rank];
    PeerCtl* ctl = ctl_of(own);
    const unsigned int e = peer_epoch(ctl), h = e & 1u;
    const int64_t half = kPeerCtlBytes / 4 + (int64_t)h * kPeerHalfFloats;
    const int G = segs.G, me = segs.rank;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthr = gridDim.x * blockDim.x;

    // 1. push
    for (int sg = 0; sg < segs.count; ++sg) {
        const int ns4 = segs.ns4[sg], units = segs.rows[sg] * ns4;
        const int64_t n4 = (int64_t)G * ns4;  // float4 per row
        float4* y = reinterpret_cast<float4*>(segs.y[sg]);
        const int64_t src0 = half + segs.off[sg];
        for (int i = tid; i < units; i += nthr) {
            const int b = i / ns4, j = i - b * ns4;
            const int64_t u = (int64_t)b * n4 + (int64_t)me * ns4 + j;  // float4 index in the segment
            const float4 v = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<float*>(own) + src0) + u);
            y[u] = v;
            for (int q = 0; q < G; ++q)
                if (q != me) reinterpret_cast<float4*>(reinterpret_cast<float*>(segs.base[q]) + src0)[u] = v;
        }
    }
    // 2. signal and wait; 3. the other ranks' columns
    if (peer_signal_wait(ctl, segs.base, me, G, h, timeout_ns, err)) {
        for (int sg = 0; sg < segs.count; ++sg) {
            const int ns4 = segs.ns4[sg], units = segs.rows[sg] * (G - 1) * ns4;
            const int64_t n4 = (int64_t)G * ns4;
            float4* y = reinterpret_cast<float4*>(segs.y[sg]);
            const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<float*>(own) + half + segs.off[sg]);
            for (int i = tid; i < units; i += nthr) {
                const int r = i / ns4, j = i - r * ns4;
                const int b = r / (G - 1), qq = r - b * (G - 1);
                const int q = qq < me ? qq : qq + 1;
                const int64_t u = (int64_t)b * n4 + (int64_t)q * ns4 + j;
                y[u] = __ldcg(src + u);
            }
        }
    }
    // 4. advance
    peer_advance(ctl, e, G);
}

// In-place all-reduce (sum) of n floats (n % 4 == 0, buf 16-byte aligned)
// over peer memory, one cooperative launch: this rank's values go into slot
// `rank` of every rank's half (16-byte stores over NVLink), then, after the
// signals, every rank adds the G slots in rank order -- the same bits on
// every rank, run to run.
struct PeerReduce {
    char* base[kMaxPeers];
    float* buf;
    int64_t n4;
    int rank, G;
};
__global__ void peer_allreduce_kernel(const __grid_constant__ PeerReduce pr, uint64_t timeout_ns, int* err) {
    char* own = pr.base[pr.rank];
    PeerCtl* ctl = ctl_of(own);
    const unsigned int e = peer_epoch(ctl), h = e & 1u;
    const int64_t half = kPeerCtlBytes / 4 + (int64_t)h * kPeerHalfFloats;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, nthr = (int64_t)gridDim.x * blockDim.x;
    float4* buf = reinterpret_cast<float4*>(pr.buf);
    const int64_t slot0 = half + (int64_t)pr.rank * pr.n4 * 4;
    for (int64_t i = tid; i < pr.n4; i += nthr) {
        const float4 v = buf[i];
        for (int q = 0; q < pr.G; ++q) reinterpret_cast<float4*>(reinterpret_cast<float*>(pr.base[q]) + slot0)[i] = v;
    }
    if (peer_signal_wait(ctl, pr.base, pr.rank, pr.G, h, timeout_ns, err)) {
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<float*>(own) + half);
        for (int64_t i = tid; i < pr.n4; i += nthr) {
            float4 a = __ldcg(src + i);
            for (int q = 1; q < pr.G; ++q) {
                const float4 b = __ldcg(src + (int64_t)q * pr.n4 + i);
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
            }
            buf[i] = a;
        }
    }
    peer_advance(ctl, e, pr.G);
}

// Launches a peer collective kernel cooperatively, one CTA per SM.
template <typename Arg>
int launch_peer(strata_ctx* ctx, void (*kern)(Arg, uint64_t, int*), const Arg& arg, cudaStream_t s, const char* what) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctx->sm_count);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, arg, (uint64_t)ctx->wait_timeout_ms * 1000000ull, ctx->err_dev);
    return check_launch(ctx, what);
}

// Orders peer work on stream s after the previous peer work (another stream).
void peer_order(strata_ctx* ctx, cudaStream_t s) {
    CommState* c = ctx->comm;
    if (c->peer_stream && c->peer_stream != s) {
        cudaEventRecord(c->order, c->peer_stream);
        cudaStreamWaitEvent(s, c->order, 0);
    }
    c->peer_stream = s;
}

// Whether this sharded GEMV takes the peer all-gather.
bool use_peer_gather(strata_ctx* ctx, const strata_weight* w, const float* x, const float* y, int batch) {
    CommState* c = ctx->comm;
    if (!c->peer_ok || c->gather_mode == STRATA_GATHER_NCCL || c->world < 2) return false;
    if ((int64_t)batch * w->rows * c->world > kPeerHalfFloats || w->rows % 4 != 0 || ((uintptr_t)y & 15)) return false;
    return gemv_peer_capable(ctx, w, x, batch);
}

// Enqueues the all-gather kernel for the pending segments (no-op when none
// are pending). Every rank flushes at the same points of the same call
// sequence, so the ranks' halves and arrival counts stay in step.
int peer_flush(strata_ctx* ctx) {
    CommState* c = ctx->comm;
    PeerPending& p = c->pending;
    if (p.segs.count == 0) return STRATA_OK;
    p.segs.rank = c->rank;
    p.segs.G = c->world;
    for (int q = 0; q < c->world; ++q) p.segs.base[q] = c->peer_base[q];
    const PeerSegs segs = p.segs;
    const cudaStream_t st = p.stream;
    p = PeerPending{};
    return launch_peer(ctx, peer_allgather_kernel, segs, st, "peer all-gather kernel");
}

// Whether the expert-parallel layer output (n floats at out) takes the peer all-reduce.
bool use_peer_reduce(strata_ctx* ctx, const float* out, int64_t n) {
    CommState* c = ctx->comm;
    return c->peer_ok && c->gather_mode != STRATA_GATHER_NCCL && c->world >= 2 && n % 4 == 0 &&
           ((uintptr_t)out & 15) == 0 && n * c->world <= kPeerHalfFloats;
}

// In-place peer all-reduce of the layer output; pending grouped gathers on
// any stream go first, so the ranks' halves stay in step.
int peer_allreduce(strata_ctx* ctx, float* buf, int64_t n, cudaStream_t s) {
    CommState* c = ctx->comm;
    int rc = peer_flush(ctx);
    if (rc) return rc;
    peer_order(ctx, s);
    PeerReduce pr{};
    for (int q = 0; q < c->world; ++q) pr.base[q] = c->peer_base[q];
    pr.buf = buf;
    pr.n4 = n / 4;
    pr.rank = c->rank;
    pr.G = c->world;
    return launch_peer(ctx, peer_allreduce_kernel, pr, s, "peer all-reduce kernel");
}

// Sharded GEMV into this rank's exchange half at the call's place; the
// all-gather kernel follows at once, or at the end of the collective group
// (one for all the group's calls on a stream).
int gemv_peer_gather(strata_ctx* ctx, const strata_weight* w, const float* x, float* y, int batch, cudaStream_t s) {
    CommState* c = ctx->comm;
    PeerPending& p = c->pending;
    const int64_t ns = w->rows, N = ns * c->world;
    const int64_t n = (int64_t)batch * N;
    int rc;
    if (p.segs.count > 0 && (p.stream != s || p.segs.count == kPeerSegs || p.floats + n > kPeerHalfFloats))
        if ((rc = peer_flush(ctx))) return rc;
    peer_order(ctx, s);
    PeerOut po{};
    po.y = data_of(c->xbuf);
    po.epoch = &ctl_of(c->xbuf)->epoch;
    po.half_floats = kPeerHalfFloats;
    po.off = p.floats + c->rank * ns;
    po.G = c->world;
    if ((rc = gemv_enqueue_strided(ctx, w, x, y + c->rank * ns, batch, N, s, &po))) return rc;
    p.stream = s;
    p.segs.y[p.segs.count] = y;
    p.segs.off[p.segs.count] = p.floats;
    p.segs.rows[p.segs.count] = batch;
    p.segs.ns4[p.segs.count] = (int)(ns / 4);
    ++p.segs.count;
    p.floats += (n + 3) & ~int64_t(3);
    return c->group_depth > 0 ? STRATA_OK : peer_flush(ctx);
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
    STRATA_CALL_RANGE();
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
    // the fused peer gather; when peer memory is unavailable only that path is off
    rc = peer_setup(ctx);
    if (rc) {
        comm_release(ctx);
        return rc;
    }
    return STRATA_OK;
}

int strata_cuda_comm_set_gather(strata_ctx* ctx, int mode) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = need_comm(ctx);
    if (rc) return rc;
    if (mode < STRATA_GATHER_AUTO || mode > STRATA_GATHER_PEER)
        return fail(ctx, STRATA_ERR_INVALID, "gather mode %d", mode);
    if (ctx->comm->group_depth > 0) return fail(ctx, STRATA_ERR_INVALID, "the gather mode cannot change inside a group");
    if (mode == STRATA_GATHER_PEER && !ctx->comm->peer_ok)
        return fail(ctx, STRATA_ERR_INVALID, "peer memory is not available on every rank");
    ctx->comm->gather_mode = mode;
    return STRATA_OK;
}

int strata_cuda_comm_peer_info(const strata_ctx* ctx, int* available, int64_t* capacity_floats) {
    if (!ctx || !available || !capacity_floats) return STRATA_ERR_INVALID;
    *available = ctx->comm && ctx->comm->peer_ok;
    *capacity_floats = *available ? kPeerHalfFloats : 0;
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
    if (--ctx->comm->group_depth == 0) {
        rc = peer_flush(ctx);
        const int rn = nccl_done(ctx, ctx->comm->comm, nccl().GroupEnd(), "ncclGroupEnd");
        return rc ? rc : rn;
    }
    return STRATA_OK;
}

int strata_cuda_gemv_sharded_dev(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                                 void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, false);
    if (rc || (rc = need_comm(ctx))) return rc;
    if (!x_dev || !y_dev) return fail(ctx, STRATA_ERR_INVALID, "null x or y");
    if (batch < 1 || batch > 8) return fail(ctx, STRATA_ERR_INVALID, "batch %d outside 1..8", batch);
    cudaSetDevice(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    CommState* c = ctx->comm;
    const int64_t ns = w->rows;
    if (use_peer_gather(ctx, w, x_dev, y_dev, batch)) return gemv_peer_gather(ctx, w, x_dev, y_dev, batch, s);
    if (c->gather_mode == STRATA_GATHER_PEER)
        return fail(ctx, STRATA_ERR_INVALID, "the peer gather does not apply to this shard (quant %u, batch %d)",
                    w->quant, batch);
    // the local GEMV writes rank r's columns of every output row in place
    // (output row pitch N = world * ns)
    if ((rc = gemv_enqueue_strided(ctx, w, x_dev, y_dev + c->rank * ns, batch, ns * c->world, s))) return rc;
    return gather_rows_inplace(ctx, y_dev, batch, ns, s);
}

int strata_cuda_gemm_sharded_dev(strata_ctx* ctx, const strata_weight* w, const uint16_t* x_dev, float* y_dev,
                                 int64_t m, void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
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
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = need_comm(ctx);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    cudaStream_t s = pick_stream(ctx, stream);
    if ((rc = moe_enqueue_checked(ctx, layer, x_dev, logits_dev, tokens, out_dev, nullptr, nullptr, s))) return rc;
    const int64_t n = tokens * moe_embd(layer);
    if (use_peer_reduce(ctx, out_dev, n)) return peer_allreduce(ctx, out_dev, n, s);
    if (ctx->comm->gather_mode == STRATA_GATHER_PEER)
        return fail(ctx, STRATA_ERR_INVALID, "the peer all-reduce does not apply to this output");
    return nccl_done(ctx, ctx->comm->comm,
                     nccl().AllReduce(out_dev, out_dev, (size_t)n, ncclFloat, ncclSum, ctx->comm->comm, s),
                     "ncclAllReduce");
}

}  // extern "C"
