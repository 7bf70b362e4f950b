// runtime.cu — contexts, resident weights and the C ABI of strata_cuda.h.
//
// The host side of the backend: it owns the CUDA stream, the pinned staging
// used by the synchronous (trait-shaped) entry points, the device workspace,
// and the weights uploaded byte-for-byte. Kernels live in the other .cu files.
#include "runtime.cuh"

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "host.h"
#include "staging.h"

using namespace strata;

namespace strata {

int fail(strata_ctx* ctx, int code, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return code;
}

int report(strata_ctx* ctx, int code, const char* msg) {
    std::lock_guard<std::mutex> g(ctx->mu);
    ctx->last_error = msg;
    return code;
}

bool quant_on_device(uint32_t quant) { return block_elems(quant) != 0; }

int cuda_fail(strata_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, e == cudaErrorMemoryAllocation ? STRATA_ERR_OOM : STRATA_ERR_CUDA, "%s: %s (%s)", what,
                cudaGetErrorString(e), cudaGetErrorName(e));
}

int64_t quant_row_bytes(uint32_t quant, int64_t cols) {
    int be = block_elems(quant), bb = block_bytes(quant);
    if (be == 0) return -1;
    return ((cols + be - 1) / be) * bb;
}

int ensure_device(strata_ctx* ctx, DevBuf& b, size_t bytes, const char* what) {
    if (b.bytes >= bytes && b.ptr) return STRATA_OK;
    if (b.ptr) {
        // the old buffer may still be read by queued work
        int rc = wait_stream(ctx, ctx->stream);
        if (rc) return rc;
        cudaFree(b.ptr);
        b.ptr = nullptr;
        b.bytes = 0;
    }
    size_t want = bytes < 4096 ? 4096 : bytes;
    ++ctx->buf_gen;
    cudaError_t e = cudaMalloc(&b.ptr, want);
    if (e != cudaSuccess) {
        b.ptr = nullptr;
        return cuda_fail(ctx, e, what);
    }
    b.bytes = want;
    return STRATA_OK;
}

int ensure_pinned(strata_ctx* ctx, PinnedBuf& b, size_t bytes, const char* what) {
    if (b.bytes >= bytes && b.ptr) return STRATA_OK;
    if (b.ptr) {
        int rc = wait_stream(ctx, ctx->stream);
        if (rc) return rc;
        cudaFreeHost(b.ptr);
        b.ptr = nullptr;
        b.dev = nullptr;
        b.bytes = 0;
    }
    size_t want = bytes < 4096 ? 4096 : bytes;
    ++ctx->buf_gen;
    cudaError_t e = cudaMallocHost(&b.ptr, want);
    if (e != cudaSuccess) {
        b.ptr = nullptr;
        return cuda_fail(ctx, e, what);
    }
    // page-locked memory is mapped into the device's address space (unified
    // addressing); kernels may read and write it in place
    if (cudaHostGetDevicePointer(&b.dev, b.ptr, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        b.dev = nullptr;
    }
    b.bytes = want;
    return STRATA_OK;
}

// Bounded wait: poll an event recorded on `s` until it completes or the
// context's timeout expires (the device work keeps running in that case; the
// context stays usable and the caller gets STRATA_ERR_TIMEOUT).
int check_device_error(strata_ctx* ctx) {
    if (ctx->err_host && *(volatile int*)ctx->err_host) {
        *(volatile int*)ctx->err_host = 0;
        return fail(ctx, STRATA_ERR_TIMEOUT, "a kernel's bounded wait expired (shared-memory copies, or the other ranks' arrivals)");
    }
    return STRATA_OK;
}

int wait_stream(strata_ctx* ctx, cudaStream_t s) {
    cudaError_t e = cudaEventRecord(ctx->done, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventRecord");
    auto t0 = std::chrono::steady_clock::now();
    int spins = 0;
    for (;;) {
        e = cudaEventQuery(ctx->done);
        if (e == cudaSuccess) return check_device_error(ctx);
        if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "device work");
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if ((uint64_t)ms > ctx->wait_timeout_ms)
            return fail(ctx, STRATA_ERR_TIMEOUT, "device work did not finish within %u ms", ctx->wait_timeout_ms);
        if (++spins > 64) std::this_thread::yield();
    }
}

cudaStream_t pick_stream(strata_ctx* ctx, void* stream) {
    return stream ? reinterpret_cast<cudaStream_t>(stream) : ctx->stream;
}

int check_launch(strata_ctx* ctx, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, what);
    return STRATA_OK;
}

int check_weight(strata_ctx* ctx, const strata_weight* w, bool expert) {
    if (!w || w->magic != kWeightMagic) return fail(ctx, STRATA_ERR_INVALID, "invalid weight handle");
    if (w->ctx != ctx) return fail(ctx, STRATA_ERR_INVALID, "weight belongs to another context");
    if (expert && w->n_expert == 0) return fail(ctx, STRATA_ERR_INVALID, "expert call on a dense tensor");
    if (!expert && w->n_expert != 0) return fail(ctx, STRATA_ERR_INVALID, "dense call on an expert tensor");
    return STRATA_OK;
}

}  // namespace strata

// ------------------------------------------------------------------ C ABI

extern "C" {

int strata_cuda_abi_version(void) { return STRATA_CUDA_ABI_VERSION; }

const char* strata_cuda_name(void) { return "cuda"; }

int strata_cuda_create(int device, strata_ctx** out) {
    if (!out) return STRATA_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return STRATA_ERR_CUDA;
    if (device < 0 || device >= n) return STRATA_ERR_INVALID;
    if (cudaSetDevice(device) != cudaSuccess) return STRATA_ERR_CUDA;
    strata_ctx* ctx = new strata_ctx();
    ctx->device = device;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        delete ctx;
        return STRATA_ERR_CUDA;
    }
    ctx->sm_count = prop.multiProcessorCount;
    ctx->l2_bytes = prop.l2CacheSize;
    ctx->cc_major = prop.major;
    ctx->cc_minor = prop.minor;
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->done, cudaEventDisableTiming) != cudaSuccess ||
        cudaHostAlloc((void**)&ctx->err_host, sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void**)&ctx->err_dev, ctx->err_host, 0) != cudaSuccess) {
        if (ctx->err_host) cudaFreeHost(ctx->err_host);
        if (ctx->done) cudaEventDestroy(ctx->done);
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
        return STRATA_ERR_CUDA;
    }
    *ctx->err_host = 0;
    *out = ctx;
    return STRATA_OK;
}

int strata_cuda_destroy(strata_ctx* ctx) {
    if (!ctx) return STRATA_ERR_INVALID;
    cudaSetDevice(ctx->device);
    int rc = wait_stream(ctx, ctx->stream);
    moe_release_all(ctx);
    comm_release(ctx);
    for (strata_weight* w : ctx->weights) {  // weights the caller did not free
        if (w->dev) cudaFree(w->dev);
        w->magic = 0;
        delete w;
    }
    ctx->weights.clear();
    for (DevBuf* b : {&ctx->x_dev, &ctx->y_dev, &ctx->work, &ctx->xfrag, &ctx->gemm_work, &ctx->x_bf16, &ctx->moe_work})
        if (b->ptr) cudaFree(b->ptr);
    for (PinnedBuf* b : {&ctx->x_host, &ctx->y_host, &ctx->stage[0], &ctx->stage[1]})
        if (b->ptr) cudaFreeHost(b->ptr);
    for (cudaEvent_t& e : ctx->stage_ev)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t& e : ctx->piece_ev)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t& e : ctx->slice_ev)
        if (e) cudaEventDestroy(e);
    if (ctx->copy) cudaStreamDestroy(ctx->copy);
    cudaEventDestroy(ctx->done);
    if (ctx->fork) cudaEventDestroy(ctx->fork);
    if (ctx->join) cudaEventDestroy(ctx->join);
    if (ctx->aux) cudaStreamDestroy(ctx->aux);
    if (ctx->aux_lo) cudaStreamDestroy(ctx->aux_lo);
    cudaStreamDestroy(ctx->stream);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    delete ctx;
    return rc;
}

const char* strata_cuda_last_error(const strata_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

int strata_cuda_set_weight_budget(strata_ctx* ctx, uint64_t bytes) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    ctx->budget_bytes = bytes;
    return STRATA_OK;
}

int strata_cuda_resident_bytes(const strata_ctx* ctx, uint64_t* out) {
    if (!ctx || !out) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(const_cast<strata_ctx*>(ctx)->mu);
    *out = ctx->resident_bytes;
    return STRATA_OK;
}

int strata_cuda_set_wait_timeout_ms(strata_ctx* ctx, uint32_t ms) {
    if (!ctx || ms == 0) return STRATA_ERR_INVALID;
    ctx->wait_timeout_ms = ms;
    return STRATA_OK;
}

int strata_cuda_set_gemv_path(strata_ctx* ctx, int path) {
    if (!ctx || path < STRATA_GEMV_AUTO || path > STRATA_GEMV_TENSOR_CORES) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    if (ctx->gemv_path != path) ++ctx->buf_gen;  // captured MoE graphs hold the old path's GEMV kernels
    ctx->gemv_path = path;
    return STRATA_OK;
}

int strata_cuda_set_gemm_terms(strata_ctx* ctx, int terms) {
    if (!ctx || terms < 1 || terms > 2) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    ctx->gemm_terms = terms;
    return STRATA_OK;
}

int strata_cuda_synchronize(strata_ctx* ctx) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    cudaSetDevice(ctx->device);
    return wait_stream(ctx, ctx->stream);
}

int strata_cuda_stream(const strata_ctx* ctx, void** out) {
    if (!ctx || !out) return STRATA_ERR_INVALID;
    *out = reinterpret_cast<void*>(ctx->stream);
    return STRATA_OK;
}

namespace {

constexpr size_t kStageChunk = size_t(32) << 20;  // bytes per staging chunk
constexpr int kStageThreads = 8;                  // host threads filling a chunk

// Bounded wait for a staging chunk's previous copy to leave the pinned buffer.
int wait_stage(strata_ctx* ctx, cudaEvent_t ev) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return STRATA_OK;
        if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "upload staging");
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if ((uint64_t)ms.count() > ctx->wait_timeout_ms)
            return fail(ctx, STRATA_ERR_TIMEOUT, "upload copy did not finish within %u ms", ctx->wait_timeout_ms);
        std::this_thread::yield();
    }
}

// Copies host byte ranges (typically slices of a read-only mmap of the model
// file, paged in on first touch) to their device destinations. Under 64 MiB
// in all: one cudaMemcpy per range. More: the ranges, taken as one stream, go
// through two pinned 32 MiB chunks; host threads fill one (taking the page
// faults in parallel) while the DMA engine drains the other, and a chunk may
// carry the end of one range and the start of the next.
int copy_in(strata_ctx* ctx, const StageSeg* segs, int64_t nseg) {
    size_t total = 0;
    for (int64_t i = 0; i < nseg; ++i) total += segs[i].n;
    if (total < 2 * kStageChunk) {
        for (int64_t i = 0; i < nseg; ++i) {
            if (!segs[i].n) continue;
            cudaError_t e = cudaMemcpy(segs[i].dst, segs[i].src, segs[i].n, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpy(weights)");
        }
        return STRATA_OK;
    }
    int rc;
    for (int k = 0; k < 2; ++k) {
        if ((rc = ensure_pinned(ctx, ctx->stage[k], kStageChunk, "cudaMallocHost(upload staging)"))) return rc;
        if (!ctx->stage_ev[k]) {
            cudaError_t e = cudaEventCreateWithFlags(&ctx->stage_ev[k], cudaEventDisableTiming);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventCreate(upload staging)");
        }
    }
    rc = STRATA_OK;
    StageCursor cur;
    std::vector<StagePiece> pieces;
    for (int i = 0;; ++i) {
        const int k = i & 1;
        const size_t len = stage_plan(segs, nseg, cur, kStageChunk, pieces);
        if (!len) break;
        if (i >= 2 && (rc = wait_stage(ctx, ctx->stage_ev[k]))) break;
        uint8_t* stage = static_cast<uint8_t*>(ctx->stage[k].ptr);
        std::thread th[kStageThreads];
        const size_t part = (len + kStageThreads - 1) / kStageThreads;
        for (int t = 0; t < kStageThreads; ++t) {
            const size_t a = t * part, b = a + part < len ? a + part : len;
            if (a >= b) continue;
            try {
                th[t] = std::thread([&pieces, segs, stage, a, b] { stage_fill(pieces, segs, stage, a, b); });
            } catch (...) {  // no thread to be had: fill this part here
                stage_fill(pieces, segs, stage, a, b);
            }
        }
        for (auto& t : th)
            if (t.joinable()) t.join();
        cudaError_t e = cudaSuccess;
        for (const StagePiece& p : pieces) {
            e = cudaMemcpyAsync(segs[p.seg].dst + p.seg_off, stage + p.off, p.n, cudaMemcpyHostToDevice,
                                ctx->stream);
            if (e != cudaSuccess) break;
        }
        if (e == cudaSuccess) e = cudaEventRecord(ctx->stage_ev[k], ctx->stream);
        if (e != cudaSuccess) {
            rc = cuda_fail(ctx, e, "cudaMemcpyAsync(weights)");
            break;
        }
    }
    if (rc) {  // copies already queued still read the pinned chunks: let them finish
        cudaStreamSynchronize(ctx->stream);
        return rc;
    }
    return wait_stream(ctx, ctx->stream);
}

// Validates one upload and returns the bytes it keeps resident (row_bytes in *rb).
int check_upload(strata_ctx* ctx, const strata_upload& u, int64_t* need, int64_t* rb) {
    const int be = block_elems(u.quant);
    if (be == 0) return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "quant type id %u is not on the CUDA path", u.quant);
    if (u.n_expert < 0 || u.rows < 0 || u.cols <= 0 || (!u.bytes && u.len > 0))
        return fail(ctx, STRATA_ERR_INVALID, "bad shape n_expert=%lld rows=%lld cols=%lld", (long long)u.n_expert,
                    (long long)u.rows, (long long)u.cols);
    if (u.cols % be != 0)
        return fail(ctx, STRATA_ERR_TRUNCATED, "cols=%lld is not a whole number of %d-element blocks",
                    (long long)u.cols, be);
    if (u.cols / be > INT64_MAX / block_bytes(u.quant))
        return fail(ctx, STRATA_ERR_INVALID, "cols=%lld is too large", (long long)u.cols);
    *rb = quant_row_bytes(u.quant, u.cols);
    const int64_t mats = u.n_expert > 0 ? u.n_expert : 1;
    if (u.rows > 0 && (mats > INT64_MAX / u.rows || mats * u.rows > INT64_MAX / *rb))
        return fail(ctx, STRATA_ERR_INVALID, "tensor of %lld x %lld rows is too large", (long long)mats,
                    (long long)u.rows);
    *need = mats * u.rows * *rb;
    if ((uint64_t)u.len < (uint64_t)*need)
        return fail(ctx, STRATA_ERR_TRUNCATED, "tensor needs %lld bytes, got %zu", (long long)*need, u.len);
    return STRATA_OK;
}

// strata_cuda_upload_many with the context lock held.
int upload_locked(strata_ctx* ctx, const strata_upload* items, int64_t n, strata_weight** out) {
    for (int64_t i = 0; i < n; ++i) out[i] = nullptr;
    std::vector<int64_t> need(n), rb(n);
    uint64_t total = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int rc = check_upload(ctx, items[i], &need[i], &rb[i]);
        if (rc) return n > 1 ? fail(ctx, rc, "upload %lld of %lld: %s", (long long)i, (long long)n,
                                   ctx->last_error.c_str())
                             : rc;
        total += (uint64_t)need[i];
    }
    if (ctx->budget_bytes && ctx->resident_bytes + total > ctx->budget_bytes)
        return fail(ctx, STRATA_ERR_BUDGET, "upload of %llu bytes exceeds the weight budget (%llu resident of %llu)",
                    (unsigned long long)total, (unsigned long long)ctx->resident_bytes,
                    (unsigned long long)ctx->budget_bytes);
    cudaSetDevice(ctx->device);
    std::vector<strata_weight*> ws(n, nullptr);
    std::vector<StageSeg> segs;
    segs.reserve(n);
    int rc = STRATA_OK;
    for (int64_t i = 0; i < n && !rc; ++i) {
        strata_weight* w = new strata_weight();
        w->ctx = ctx;
        w->quant = items[i].quant;
        w->n_expert = items[i].n_expert;
        w->rows = items[i].rows;
        w->cols = items[i].cols;
        w->row_bytes = rb[i];
        w->bytes = (size_t)need[i];
        ws[i] = w;
        if (need[i] > 0) {
            cudaError_t e = cudaMalloc(&w->dev, (size_t)need[i]);
            if (e != cudaSuccess)
                rc = cuda_fail(ctx, e, "cudaMalloc(weights)");
            else
                segs.push_back({w->dev, items[i].bytes, (size_t)need[i]});
        }
    }
    if (!rc) rc = copy_in(ctx, segs.data(), (int64_t)segs.size());
    if (rc) {
        for (strata_weight* w : ws) {
            if (w && w->dev) cudaFree(w->dev);
            delete w;
        }
        return rc;
    }
    for (int64_t i = 0; i < n; ++i) {
        strata_weight* w = ws[i];
        if (w->n_expert == 0 && w->bytes > 0)
            w->has_tmap = encode_gemv_tmap(w->quant, w->dev, w->rows, w->row_bytes, w->tmap);
        out[i] = w;
        ctx->weights.insert(w);
    }
    ctx->resident_bytes += total;
    return STRATA_OK;
}

}  // namespace

int strata_cuda_upload(strata_ctx* ctx, const uint8_t* bytes, size_t len, uint32_t quant, int64_t n_expert,
                       int64_t rows, int64_t cols, strata_weight** out) {
    if (!ctx || !out) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    const strata_upload u{bytes, len, quant, n_expert, rows, cols};
    return upload_locked(ctx, &u, 1, out);
}

int strata_cuda_upload_many(strata_ctx* ctx, const strata_upload* items, int64_t n, strata_weight** out) {
    if (!ctx || n < 0 || (n > 0 && (!items || !out))) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    return upload_locked(ctx, items, n, out);
}

int strata_cuda_free_weight(strata_weight* w) {
    if (!w || w->magic != kWeightMagic) return STRATA_ERR_INVALID;
    strata_ctx* ctx = w->ctx;
    std::lock_guard<std::mutex> g(ctx->mu);
    cudaSetDevice(ctx->device);
    int rc = wait_stream(ctx, ctx->stream);
    if (w->dev) cudaFree(w->dev);
    ctx->resident_bytes -= (uint64_t)w->bytes;
    ctx->weights.erase(w);
    w->magic = 0;
    delete w;
    return rc;
}

int strata_cuda_dequant(strata_ctx* ctx, const strata_weight* w, int64_t expert, int64_t row0, int64_t nrows,
                        float* out_host) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    if (!w || w->magic != kWeightMagic || w->ctx != ctx) return fail(ctx, STRATA_ERR_INVALID, "invalid weight handle");
    int64_t mats = w->n_expert > 0 ? w->n_expert : 1;
    if (expert < 0 || expert >= mats || row0 < 0 || nrows < 0 || row0 + nrows > w->rows || (!out_host && nrows))
        return fail(ctx, STRATA_ERR_INVALID, "dequant range out of bounds");
    if (nrows == 0) return STRATA_OK;
    cudaSetDevice(ctx->device);
    size_t nbytes = (size_t)(nrows * w->cols) * sizeof(float);
    int rc = ensure_device(ctx, ctx->y_dev, nbytes, "cudaMalloc(dequant out)");
    if (!rc) rc = ensure_pinned(ctx, ctx->y_host, nbytes, "cudaMallocHost(dequant out)");
    if (rc) return rc;
    const uint8_t* base = w->dev + (expert * w->rows + row0) * w->row_bytes;
    if (launch_dequant(w->quant, base, w->row_bytes, w->cols, nrows, (float*)ctx->y_dev.ptr, ctx->stream))
        return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "no dequant kernel for quant %u", w->quant);
    if ((rc = check_launch(ctx, "dequant kernel"))) return rc;
    cudaError_t e = cudaMemcpyAsync(ctx->y_host.ptr, ctx->y_dev.ptr, nbytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(D2H)");
    if ((rc = wait_stream(ctx, ctx->stream))) return rc;
    copy_host(out_host, ctx->y_host.ptr, nbytes);
    return STRATA_OK;
}

// ---- decode GEMV

}  // extern "C"

namespace strata {

// Waits (bounded, like wait_stream) for an event already recorded.
static int wait_event(strata_ctx* ctx, cudaEvent_t ev) {
    auto t0 = std::chrono::steady_clock::now();
    int spins = 0;
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return STRATA_OK;
        if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "device work");
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if ((uint64_t)ms > ctx->wait_timeout_ms)
            return fail(ctx, STRATA_ERR_TIMEOUT, "device work did not finish within %u ms", ctx->wait_timeout_ms);
        if (++spins > 64) std::this_thread::yield();
    }
}

// The result of the work queued on the context stream, `bytes` at `src_dev`,
// into the caller's buffer: in pieces of at least 2 MiB (up to kPieces),
// each copied device -> pinned staging -> caller, the host copy of piece k
// overlapping the transfer of piece k + 1; returns once every byte is out.
// (Each transfer has ~10-15 us of fixed latency, which smaller pieces would
// add up to more than the overlap saves.)
int copy_out(strata_ctx* ctx, void* dst, const void* src_dev, size_t bytes) {
    constexpr size_t kMinPiece = size_t(2) << 20;
    size_t np = (bytes + kMinPiece - 1) / kMinPiece;
    np = np < 1 ? 1 : (np > (size_t)strata_ctx::kPieces ? (size_t)strata_ctx::kPieces : np);
    const size_t piece = ((bytes + np - 1) / np + 255) & ~size_t(255);
    for (size_t k = 0; k < np; ++k)
        if (!ctx->piece_ev[k]) {
            cudaError_t e = cudaEventCreateWithFlags(&ctx->piece_ev[k], cudaEventDisableTiming);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventCreate(result pieces)");
        }
    char* h = static_cast<char*>(ctx->y_host.ptr);
    const char* d = static_cast<const char*>(src_dev);
    if (bytes >= CopyPool::kMin) ctx->copy_pool.prime();  // threads ready when the first piece lands
    size_t issued = 0;
    for (size_t k = 0; k < np && issued < bytes; ++k) {
        const size_t len = issued + piece < bytes ? piece : bytes - issued;
        cudaError_t e = cudaMemcpyAsync(h + issued, d + issued, len, cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaEventRecord(ctx->piece_ev[k], ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(D2H)");
        issued += len;
    }
    size_t done = 0;
    for (size_t k = 0; k < np && done < bytes; ++k) {
        const size_t len = done + piece < bytes ? piece : bytes - done;
        int rc = wait_event(ctx, ctx->piece_ev[k]);
        if (rc) return rc;
        if (k == 0 && (rc = check_device_error(ctx))) return rc;
        ctx->copy_pool.copy(static_cast<char*>(dst) + done, h + done, len);
        done += len;
    }
    return check_device_error(ctx);
}

// A host-buffer GEMV whose result is too large to store in place: the rows
// are cut into up to kPieces slices (whole rounds of 16-row tiles over the
// SMs at two or three CTAs each; a short last slice), computed one after
// another on the context stream (the activation prologue once, the slices
// reusing its limbs). Each slice's rows of every token are copied device ->
// pinned on the copy stream as soon as that slice is done, overlapping the
// next slices' compute, and pinned -> caller by the pool's threads while the
// next slice transfers. Returns once every byte is out.
static int gemv_sliced_out(strata_ctx* ctx, const strata_weight* w, const float* xd, float* y, int batch) {
    const int64_t N = w->rows;
    const size_t yb = (size_t)batch * (size_t)N * sizeof(float);
    constexpr size_t kMinSlice = size_t(512) << 10;
    int S = (int)(yb / kMinSlice);
    S = S < 1 ? 1 : (S > strata_ctx::kPieces ? strata_ctx::kPieces : S);
    const int64_t unit = (int64_t)16 * ctx->sm_count * 6;
    int64_t rs = (N + S - 1) / S;
    rs = (rs + unit - 1) / unit * unit;
    if (!ctx->copy) {
        cudaError_t e = cudaStreamCreateWithFlags(&ctx->copy, cudaStreamNonBlocking);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamCreate(result copies)");
    }
    for (int k = 0; k < strata_ctx::kPieces; ++k)
        for (cudaEvent_t* ev : {&ctx->slice_ev[k], &ctx->piece_ev[k]})
            if (!*ev) {
                cudaError_t e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
                if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventCreate(result slices)");
            }
    int rc = ensure_device(ctx, ctx->xfrag, (size_t)std::max<int64_t>(gemv_mma_work_bytes(w->cols, batch), 4 << 20),
                           "cudaMalloc(x limbs)");
    if (rc) return rc;
    char* h = static_cast<char*>(ctx->y_host.ptr);
    char* d = static_cast<char*>(ctx->y_dev.ptr);
    const size_t pitch = (size_t)N * sizeof(float);
    int issued = 0;
    bool copying = false;  // a slice's copy is queued on the copy stream
    // on an error after a slice's copy was queued, it may still be writing
    // the pinned staging: wait (bounded) for it before returning
    auto bail = [&](int code) {
        if (copying) {
            const std::string why = ctx->last_error;
            (void)wait_stream(ctx, ctx->copy);
            ctx->last_error = why;
        }
        return code;
    };
    for (int64_t r0 = 0; r0 < N; r0 += rs, ++issued) {
        const int64_t r1 = std::min(N, r0 + rs);
        alignas(64) unsigned char tm[128];
        const uint8_t* base = w->dev + r0 * w->row_bytes;
        const bool has_tm = w->has_tmap && encode_gemv_tmap(w->quant, base, r1 - r0, w->row_bytes, tm);
        GemvArgs a{base, w->row_bytes, r1 - r0, w->cols, xd, reinterpret_cast<float*>(d) + r0, batch, ctx->sm_count,
                   has_tm ? tm : nullptr, N, nullptr};
        launch_gemv_mma(w->quant, a, ctx->xfrag.ptr, ctx->err_dev, ctx->stream, issued == 0);
        if ((rc = check_launch(ctx, "tensor-core gemv kernel (slice)"))) return bail(rc);
        const size_t off = (size_t)r0 * sizeof(float), width = (size_t)(r1 - r0) * sizeof(float);
        cudaError_t e = cudaEventRecord(ctx->slice_ev[issued], ctx->stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->copy, ctx->slice_ev[issued], 0);
        if (e == cudaSuccess) {
            e = cudaMemcpy2DAsync(h + off, pitch, d + off, pitch, width, (size_t)batch, cudaMemcpyDeviceToHost,
                                  ctx->copy);
            copying = copying || e == cudaSuccess;
        }
        if (e == cudaSuccess) e = cudaEventRecord(ctx->piece_ev[issued], ctx->copy);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "result slice copy"));
    }
    ctx->copy_pool.prime();  // threads ready when the first slice lands
    for (int k = 0; k < issued; ++k) {
        const int64_t r0 = k * rs, r1 = std::min(N, r0 + rs);
        if ((rc = wait_event(ctx, ctx->piece_ev[k]))) return bail(rc);
        if ((rc = check_device_error(ctx))) return bail(rc);
        const size_t off = (size_t)r0 * sizeof(float);
        ctx->copy_pool.copy2d(reinterpret_cast<char*>(y) + off, pitch, h + off, pitch,
                              (size_t)(r1 - r0) * sizeof(float), (size_t)batch);
    }
    return STRATA_OK;
}

int gemv_enqueue(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                 cudaStream_t s) {
    return gemv_enqueue_strided(ctx, w, x_dev, y_dev, batch, 0, s);
}

// Whether the GEMV of w at this batch runs on the tensor-core path (the
// only one with the fused peer-store epilogue).
bool gemv_peer_capable(strata_ctx* ctx, const strata_weight* w, const float* x_dev, int batch) {
    GemvArgs a{w->dev, w->row_bytes, w->rows, w->cols, x_dev, nullptr, batch, ctx->sm_count,
               w->has_tmap ? w->tmap : nullptr};
    return ctx->gemv_path != STRATA_GEMV_CUDA_CORES && gemv_mma_supported(w->quant, a);
}

// y row b at y_dev + b * ldy (ldy 0: rows are w->rows floats apart). With
// `peers` the outputs go to this rank's exchange buffer instead (tensor-core
// path only).
int gemv_enqueue_strided(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                         int64_t ldy, cudaStream_t s, const PeerOut* peers) {
    if (batch < 1 || batch > 8) return fail(ctx, STRATA_ERR_INVALID, "batch %d outside 1..8", batch);
    if (((uintptr_t)x_dev & 15) || ((uintptr_t)y_dev & 3))
        return fail(ctx, STRATA_ERR_INVALID, "x must be 16-byte and y 4-byte aligned");
    GemvArgs a{w->dev, w->row_bytes, w->rows, w->cols, x_dev, y_dev, batch, ctx->sm_count,
               w->has_tmap ? w->tmap : nullptr, ldy, peers};
    if (ctx->gemv_path != STRATA_GEMV_CUDA_CORES && gemv_mma_supported(w->quant, a)) {
        int64_t need = gemv_mma_work_bytes(w->cols, batch);
        int rc = ensure_device(ctx, ctx->xfrag, (size_t)(need > (4 << 20) ? need : (4 << 20)), "cudaMalloc(x limbs)");
        if (rc) return rc;
        launch_gemv_mma(w->quant, a, ctx->xfrag.ptr, ctx->err_dev, s);
        return check_launch(ctx, "tensor-core gemv kernel");
    }
    if (peers) return fail(ctx, STRATA_ERR_INVALID, "the peer-store epilogue needs the tensor-core gemv");
    if (ctx->gemv_path == STRATA_GEMV_TENSOR_CORES)
        return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "no tensor-core gemv for quant %u", w->quant);
    if (w->quant == kQ8_0 && gemv_q8_0_bulk_supported(a)) {
        launch_gemv_q8_0_bulk(a, ctx->err_dev, s);
        return check_launch(ctx, "q8_0 gemv kernel");
    }
    if (launch_gemv(w->quant, a, s))
        return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "no gemv kernel for quant %u", w->quant);
    return check_launch(ctx, "gemv kernel");
}

}  // namespace strata

extern "C" {

int strata_cuda_gemv_dev(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int batch,
                         void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, false);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return gemv_enqueue(ctx, w, x_dev, y_dev, batch, pick_stream(ctx, stream));
}

int strata_cuda_gemv(strata_ctx* ctx, const strata_weight* w, const float* x, float* y, int batch) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, false);
    if (rc) return rc;
    if (!x || !y) return fail(ctx, STRATA_ERR_INVALID, "null x or y");
    if (batch < 1 || batch > 8) return fail(ctx, STRATA_ERR_INVALID, "batch %d outside 1..8", batch);
    cudaSetDevice(ctx->device);
    size_t xb = (size_t)batch * (size_t)w->cols * sizeof(float);
    size_t yb = (size_t)batch * (size_t)w->rows * sizeof(float);
    if ((rc = ensure_device(ctx, ctx->x_dev, xb, "cudaMalloc(x)"))) return rc;
    if ((rc = ensure_device(ctx, ctx->y_dev, yb, "cudaMalloc(y)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->x_host, xb, "cudaMallocHost(x)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->y_host, yb, "cudaMallocHost(y)"))) return rc;
    ctx->copy_pool.copy(ctx->x_host.ptr, x, xb);
    // On the tensor-core path x is read once, by the activation prologue: it
    // reads the pinned staging in place (no copy of its own). The CUDA-core
    // kernels re-read x per row, so they get a device copy.
    const float* xd = static_cast<const float*>(ctx->x_host.dev);
    if (!xd || !gemv_peer_capable(ctx, w, xd, batch)) {
        cudaError_t e = cudaMemcpyAsync(ctx->x_dev.ptr, ctx->x_host.ptr, xb, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(H2D)");
        xd = static_cast<const float*>(ctx->x_dev.ptr);
    }
    // A result of up to 1 MiB is stored by the GEMV straight into the pinned
    // staging (each value written once; no transfer to wait for), larger ones
    // go through device memory and the pieced copy-out.
    constexpr size_t kInPlaceOut = size_t(1) << 20;
    if (yb > kInPlaceOut && xd == ctx->x_host.dev) return gemv_sliced_out(ctx, w, xd, y, batch);
    float* yd = yb <= kInPlaceOut ? static_cast<float*>(ctx->y_host.dev) : nullptr;
    if ((rc = gemv_enqueue(ctx, w, xd, yd ? yd : (float*)ctx->y_dev.ptr, batch, ctx->stream))) return rc;
    if (!yd) return copy_out(ctx, y, ctx->y_dev.ptr, yb);
    if (!ctx->piece_ev[0]) {
        cudaError_t e = cudaEventCreateWithFlags(&ctx->piece_ev[0], cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventCreate(result pieces)");
    }
    cudaError_t e = cudaEventRecord(ctx->piece_ev[0], ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventRecord(result)");
    if ((rc = wait_event(ctx, ctx->piece_ev[0]))) return rc;
    if ((rc = check_device_error(ctx))) return rc;
    ctx->copy_pool.copy(y, ctx->y_host.ptr, yb);
    return STRATA_OK;
}

// ---- prefill GEMM

}  // extern "C"

namespace strata {

int gemm_enqueue(strata_ctx* ctx, const strata_weight* w, const uint16_t* x_dev, float* y_dev, int64_t m,
                 cudaStream_t s) {
    if (m < 1 || m >= (1ll << 31)) return fail(ctx, STRATA_ERR_INVALID, "m %lld outside 1..2^31-1", (long long)m);
    if (((uintptr_t)x_dev & 15) || ((uintptr_t)y_dev & 15))
        return fail(ctx, STRATA_ERR_INVALID, "x and y must be 16-byte aligned");
    GemmArgs a{w->dev, w->row_bytes, w->rows, w->cols, x_dev, y_dev, m, ctx->gemm_terms, ctx->sm_count,
               ctx->err_dev, nullptr};
    if (!gemm_tc_supported(w->quant, a)) {
        if (w->quant != kQ4_K && w->quant != kQ5_K && w->quant != kQ6_K)
            return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "no prefill gemm for quant %u", w->quant);
        return fail(ctx, STRATA_ERR_INVALID, "prefill gemm needs cols %% 256 == 0 and 16-byte rows (cols %lld)",
                    (long long)w->cols);
    }
    const int64_t wf = gemm_tc_work_floats(a);
    if (wf > 0) {
        int rc = ensure_device(ctx, ctx->gemm_work, (size_t)wf * sizeof(float), "cudaMalloc(gemm split-K)");
        if (rc) return rc;
        a.work = (float*)ctx->gemm_work.ptr;
    }
    int k = launch_gemm_tc(w->quant, a, s);
    if (k) return fail(ctx, STRATA_ERR_CUDA, "prefill gemm launch setup failed (%d)", k);
    return check_launch(ctx, "prefill gemm kernel");
}

}  // namespace strata

extern "C" {

static int gemm_check(strata_ctx* ctx, const strata_weight* w, const void* x, const void* y) {
    int rc = check_weight(ctx, w, false);
    if (rc) return rc;
    if (!x || !y) return fail(ctx, STRATA_ERR_INVALID, "null x or y");
    return STRATA_OK;
}

int strata_cuda_gemm_bf16_dev(strata_ctx* ctx, const strata_weight* w, const uint16_t* x_dev, float* y_dev,
                              int64_t m, void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = gemm_check(ctx, w, x_dev, y_dev);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return gemm_enqueue(ctx, w, x_dev, y_dev, m, pick_stream(ctx, stream));
}

int strata_cuda_gemm_f32_dev(strata_ctx* ctx, const strata_weight* w, const float* x_dev, float* y_dev, int64_t m,
                             void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = gemm_check(ctx, w, x_dev, y_dev);
    if (rc) return rc;
    if (m < 1 || m >= (1ll << 31)) return fail(ctx, STRATA_ERR_INVALID, "m %lld outside 1..2^31-1", (long long)m);
    cudaSetDevice(ctx->device);
    const int64_t n = m * w->cols;
    if ((rc = ensure_device(ctx, ctx->x_bf16, (size_t)n * 2, "cudaMalloc(x bf16)"))) return rc;
    cudaStream_t s = pick_stream(ctx, stream);
    launch_f32_to_bf16(x_dev, (uint16_t*)ctx->x_bf16.ptr, n, ctx->sm_count, s);
    if ((rc = check_launch(ctx, "bf16 rounding kernel"))) return rc;
    return gemm_enqueue(ctx, w, (const uint16_t*)ctx->x_bf16.ptr, y_dev, m, s);
}

// Host-buffer GEMM: pinned staging, H2D, optional f32 -> bf16 rounding, GEMM, D2H, bounded wait.
static int gemm_host(strata_ctx* ctx, const strata_weight* w, const void* x, size_t x_elem, float* y, int64_t m) {
    if (!ctx) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = gemm_check(ctx, w, x, y);
    if (rc) return rc;
    if (m < 1 || m >= (1ll << 31)) return fail(ctx, STRATA_ERR_INVALID, "m %lld outside 1..2^31-1", (long long)m);
    cudaSetDevice(ctx->device);
    const size_t xb = (size_t)m * (size_t)w->cols * x_elem;
    const size_t yb = (size_t)m * (size_t)w->rows * sizeof(float);
    if ((rc = ensure_device(ctx, ctx->x_dev, xb, "cudaMalloc(x)"))) return rc;
    if ((rc = ensure_device(ctx, ctx->y_dev, yb, "cudaMalloc(y)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->x_host, xb, "cudaMallocHost(x)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->y_host, yb, "cudaMallocHost(y)"))) return rc;
    const uint16_t* xg = (const uint16_t*)ctx->x_dev.ptr;
    if (x_elem == 4) {
        const size_t nb = (size_t)m * (size_t)w->cols * 2;
        if ((rc = ensure_device(ctx, ctx->x_bf16, nb, "cudaMalloc(x bf16)"))) return rc;
        xg = (const uint16_t*)ctx->x_bf16.ptr;
    }
    copy_host(ctx->x_host.ptr, x, xb);
    cudaError_t e = cudaMemcpyAsync(ctx->x_dev.ptr, ctx->x_host.ptr, xb, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(H2D)");
    if (x_elem == 4) {
        launch_f32_to_bf16((const float*)ctx->x_dev.ptr, (uint16_t*)ctx->x_bf16.ptr, m * w->cols, ctx->sm_count,
                           ctx->stream);
        if ((rc = check_launch(ctx, "bf16 rounding kernel"))) return rc;
    }
    if ((rc = gemm_enqueue(ctx, w, xg, (float*)ctx->y_dev.ptr, m, ctx->stream))) return rc;
    e = cudaMemcpyAsync(ctx->y_host.ptr, ctx->y_dev.ptr, yb, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(D2H)");
    if ((rc = wait_stream(ctx, ctx->stream))) return rc;
    copy_host(y, ctx->y_host.ptr, yb);
    return STRATA_OK;
}

int strata_cuda_gemm_bf16(strata_ctx* ctx, const strata_weight* w, const uint16_t* x, float* y, int64_t m) {
    STRATA_CALL_RANGE();
    return gemm_host(ctx, w, x, 2, y, m);
}

int strata_cuda_gemm_f32(strata_ctx* ctx, const strata_weight* w, const float* x, float* y, int64_t m) {
    STRATA_CALL_RANGE();
    return gemm_host(ctx, w, x, 4, y, m);
}

// ---- expert GEMV

static int expert_enqueue(strata_ctx* ctx, const strata_weight* w, int64_t e, const float* x_dev, float* y_dev,
                          int batch, cudaStream_t s) {
    if (e < 0 || e >= w->n_expert) return fail(ctx, STRATA_ERR_INVALID, "expert %lld out of range", (long long)e);
    if (batch < 1 || batch > 64) return fail(ctx, STRATA_ERR_INVALID, "batch %d outside 1..64", batch);
    int64_t wf = expert_gemv_work_floats(w->rows, w->cols, ctx->sm_count);
    int rc = ensure_device(ctx, ctx->work, (size_t)wf * sizeof(float), "cudaMalloc(workspace)");
    if (rc) return rc;
    ExpertGemvArgs a{w->dev + e * w->rows * w->row_bytes, w->row_bytes, w->rows, w->cols, x_dev, y_dev, batch,
                     ctx->sm_count};
    int k = launch_expert_gemv_ws(w->quant, a, (float*)ctx->work.ptr, wf, s);
    if (k) return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "no expert gemv kernel for quant %u (%d)", w->quant, k);
    return check_launch(ctx, "expert gemv kernel");
}

int strata_cuda_expert_gemv_dev(strata_ctx* ctx, const strata_weight* w, int64_t e, const float* x_dev,
                                float* y_dev, int batch, void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, true);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return expert_enqueue(ctx, w, e, x_dev, y_dev, batch, pick_stream(ctx, stream));
}

int strata_cuda_expert_gemv(strata_ctx* ctx, const strata_weight* w, int64_t e, const float* x, float* y,
                            int batch) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_weight(ctx, w, true);
    if (rc) return rc;
    if (!x || !y) return fail(ctx, STRATA_ERR_INVALID, "null x or y");
    if (batch < 1 || batch > 64) return fail(ctx, STRATA_ERR_INVALID, "batch %d outside 1..64", batch);
    cudaSetDevice(ctx->device);
    size_t xb = (size_t)batch * (size_t)w->rows * sizeof(float);
    size_t yb = (size_t)batch * (size_t)w->cols * sizeof(float);
    if ((rc = ensure_device(ctx, ctx->x_dev, xb, "cudaMalloc(x)"))) return rc;
    if ((rc = ensure_device(ctx, ctx->y_dev, yb, "cudaMalloc(y)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->x_host, xb, "cudaMallocHost(x)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->y_host, yb, "cudaMallocHost(y)"))) return rc;
    copy_host(ctx->x_host.ptr, x, xb);
    cudaError_t err = cudaMemcpyAsync(ctx->x_dev.ptr, ctx->x_host.ptr, xb, cudaMemcpyHostToDevice, ctx->stream);
    if (err != cudaSuccess) return cuda_fail(ctx, err, "cudaMemcpyAsync(H2D)");
    if ((rc = expert_enqueue(ctx, w, e, (const float*)ctx->x_dev.ptr, (float*)ctx->y_dev.ptr, batch, ctx->stream)))
        return rc;
    err = cudaMemcpyAsync(ctx->y_host.ptr, ctx->y_dev.ptr, yb, cudaMemcpyDeviceToHost, ctx->stream);
    if (err != cudaSuccess) return cuda_fail(ctx, err, "cudaMemcpyAsync(D2H)");
    if ((rc = wait_stream(ctx, ctx->stream))) return rc;
    copy_host(y, ctx->y_host.ptr, yb);
    return STRATA_OK;
}

}  // extern "C"
