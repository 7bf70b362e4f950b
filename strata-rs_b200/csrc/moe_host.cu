// moe_host.cu — the C ABI of the device MoE layer (strata_cuda_moe_*).
//
// A strata_moe holds the uploaded weight handles of one layer
// (strata_core::moe::MoeLayer, crates/strata-core/src/moe.rs:22-35) and the
// expert range this context owns; strata_cuda_moe_ffn plans the launch for
// the token count (grid slots, row chunks, workspace layout) and enqueues the
// kernels of moe.cu on the context's stream or the caller's.
#include <cstring>

#include "moe.cuh"
#include "runtime.cuh"

using namespace strata;

// A host-buffer call of the layer captured as one CUDA graph (the input
// copy, the layer's launches on both streams, the output copy) for a token
// count, valid while the context's buffers are those of generation `gen`.
struct MoeGraph {
    int64_t T = 0;
    bool logits = false;
    uint64_t gen = 0;
    cudaGraphExec_t exec = nullptr;
    uint64_t used = 0;
};

struct strata_moe {
    uint32_t magic = 0x454F4D53u;  // "SMOE"
    strata_ctx* ctx = nullptr;
    strata_moe_desc d{};
    static constexpr int kGraphs = 4;  // token counts kept (least recently used replaced)
    mutable MoeGraph graphs[kGraphs];
    mutable uint64_t tick = 0;
};

namespace {

constexpr uint32_t kMoeMagic = 0x454F4D53u;

MoeTensor tensor_of(const strata_weight* w) {
    MoeTensor t;
    if (!w) return t;
    t.quant = w->quant;
    t.W = w->dev;
    t.row_bytes = w->row_bytes;
    t.expert_bytes = w->rows * w->row_bytes;
    t.tmap = w->has_tmap ? w->tmap : nullptr;
    return t;
}

int check_dense(strata_ctx* ctx, const strata_weight* w, int64_t rows, int64_t cols, const char* name) {
    if (!w) return fail(ctx, STRATA_ERR_INVALID, "moe: %s is missing", name);
    int rc = check_weight(ctx, w, false);
    if (rc) return rc;
    if (w->n_expert != 0 || w->rows != rows || w->cols != cols)
        return fail(ctx, STRATA_ERR_INVALID, "moe: %s is %lldx%lld (experts %lld), want %lldx%lld", name,
                    (long long)w->rows, (long long)w->cols, (long long)w->n_expert, (long long)rows, (long long)cols);
    return STRATA_OK;  // every uploadable type has a dense GEMV
}

int check_experts(strata_ctx* ctx, const strata_weight* w, int64_t held, int64_t rows, int64_t cols,
                  const char* name) {
    if (!w) return fail(ctx, STRATA_ERR_INVALID, "moe: %s is missing", name);
    int rc = check_weight(ctx, w, true);
    if (rc) return rc;
    if (w->n_expert != held || w->rows != rows || w->cols != cols)
        return fail(ctx, STRATA_ERR_INVALID, "moe: %s is [%lld][%lld][%lld], want [%lld][%lld][%lld]", name,
                    (long long)w->n_expert, (long long)w->rows, (long long)w->cols, (long long)held,
                    (long long)rows, (long long)cols);
    if (!moe_expert_quant_supported(w->quant))
        return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "moe: %s quant %u has no grouped kernel", name, w->quant);
    if (cols % 256 != 0)
        return fail(ctx, STRATA_ERR_INVALID, "moe: %s columns %lld are not a multiple of 256", name,
                    (long long)cols);
    return STRATA_OK;
}

int moe_enqueue(strata_ctx* ctx, const strata_moe* L, const float* x, const float* logits, int64_t T, float* out,
                int32_t* ids, float* wts, cudaStream_t s) {
    const strata_moe_desc& d = L->d;
    if (T < 1 || T * d.top_k > (1 << 24)) return fail(ctx, STRATA_ERR_INVALID, "moe: tokens %lld", (long long)T);
    if (!logits && !d.router) return fail(ctx, STRATA_ERR_INVALID, "moe: no router logits and no router weight");
    MoePlan p{};
    p.T = (int)T;
    p.E = (int)d.n_expert;
    p.k = (int)d.top_k;
    p.n_embd = (int)d.n_embd;
    p.n_ff = (int)d.n_ff;
    p.n_ff_s = (int)d.n_ff_shexp;
    p.e_begin = (int)d.expert_begin;
    p.e_end = (int)d.expert_end;
    p.shared = d.with_shared && d.gate_shexp;
    p.need_router = logits == nullptr;
    const int64_t held = d.expert_end - d.expert_begin;
    p.slots = (int)(T * d.top_k < held ? T * d.top_k : held);
    p.sm_count = ctx->sm_count;
    p.rc_gu = moe_row_chunks(p.slots, 2, p.n_embd, p.sm_count, p.T);
    p.rc_d = moe_row_chunks(p.slots, 1, p.n_ff, p.sm_count, p.T);
    MoeWork layout = moe_work_layout(p);
    int rc = ensure_device(ctx, ctx->moe_work, (size_t)layout.bytes, "cudaMalloc(moe workspace)");
    if (rc) return rc;
    MoeLaunch ml{};
    ml.plan = p;
    ml.layout = layout;
    ml.work = ctx->moe_work.ptr;
    ml.x = x;
    ml.logits = logits;
    ml.out = out;
    ml.ids_out = reinterpret_cast<int*>(ids);
    ml.wts_out = wts;
    ml.err = ctx->err_dev;
    ml.router = tensor_of(d.router);
    ml.gate = tensor_of(d.gate_exps);
    ml.up = tensor_of(d.up_exps);
    ml.down = tensor_of(d.down_exps);
    ml.gate_s = tensor_of(d.gate_shexp);
    ml.up_s = tensor_of(d.up_shexp);
    ml.down_s = tensor_of(d.down_shexp);
    ml.gate_inp_s = tensor_of(d.gate_inp_shexp);
    ml.aux = T <= 2 ? ctx->aux : ctx->aux_lo;
    ml.fork = ctx->fork;
    ml.join = ctx->join;
    int k = launch_moe_layer(ml, s);
    if (k) return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "moe: no kernel for a tensor's quant type (%d)", k);
    return check_launch(ctx, "moe layer kernels");
}

// Captures `enqueue` (the whole host-buffer call on the context stream) into
// a graph for token count T, replacing the least recently used entry. Best
// effort: when the capture or the instantiation fails the call simply stays
// uncached (the error is cleared; the direct path has already run).
template <typename F>
void capture_layer(strata_ctx* ctx, const strata_moe* L, int64_t T, bool logits, F&& enqueue) {
    MoeGraph* slot = &L->graphs[0];
    for (MoeGraph& m : L->graphs)
        if (!m.exec || m.used < slot->used) slot = &m;
    if (slot->exec) cudaGraphExecDestroy(slot->exec);
    *slot = MoeGraph{};
    const uint64_t gen = ctx->buf_gen;
    if (cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        (void)cudaGetLastError();
        return;
    }
    const std::string saved = ctx->last_error;
    const int rc = enqueue();
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (rc == STRATA_OK && e == cudaSuccess && g && ctx->buf_gen == gen &&
        cudaGraphInstantiate(&exec, g, 0) == cudaSuccess) {
        slot->T = T;
        slot->logits = logits;
        slot->gen = gen;
        slot->exec = exec;
        slot->used = ++L->tick;
    }
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
    ctx->last_error = saved;
}

void release_graphs(const strata_moe* L) {
    for (MoeGraph& m : L->graphs) {
        if (m.exec) cudaGraphExecDestroy(m.exec);
        m = MoeGraph{};
    }
}

int check_moe(strata_ctx* ctx, const strata_moe* L) {
    if (!L || L->magic != kMoeMagic) return fail(ctx, STRATA_ERR_INVALID, "invalid moe layer handle");
    if (L->ctx != ctx) return fail(ctx, STRATA_ERR_INVALID, "moe layer belongs to another context");
    return STRATA_OK;
}

}  // namespace

namespace strata {

void moe_release_all(strata_ctx* ctx) {
    for (strata_moe* L : ctx->moes) {
        release_graphs(L);
        L->ctx = nullptr;
    }
    ctx->moes.clear();
}

int moe_enqueue_checked(strata_ctx* ctx, const strata_moe* L, const float* x, const float* logits, int64_t T,
                        float* out, int32_t* ids, float* wts, cudaStream_t s) {
    int rc = check_moe(ctx, L);
    if (rc) return rc;
    if (!x || !out) return fail(ctx, STRATA_ERR_INVALID, "moe: null x or out");
    return moe_enqueue(ctx, L, x, logits, T, out, ids, wts, s);
}

int64_t moe_embd(const strata_moe* L) { return L->d.n_embd; }

}  // namespace strata

extern "C" {

int strata_cuda_moe_create(strata_ctx* ctx, const strata_moe_desc* d, strata_moe** out) {
    if (!ctx || !d || !out) return STRATA_ERR_INVALID;
    std::lock_guard<std::mutex> g(ctx->mu);
    *out = nullptr;
    if (d->n_embd <= 0 || d->n_expert <= 0 || d->n_expert > 1024 || d->top_k <= 0 || d->top_k > 32 ||
        d->n_ff <= 0 || d->n_embd % 256 != 0 || d->n_ff % 256 != 0)
        return fail(ctx, STRATA_ERR_INVALID,
                    "moe: need n_embd, n_ff multiples of 256, 1 <= n_expert <= 1024, 1 <= top_k <= 32");
    if (d->expert_begin < 0 || d->expert_end > d->n_expert || d->expert_begin >= d->expert_end)
        return fail(ctx, STRATA_ERR_INVALID, "moe: expert range [%lld, %lld) of %lld", (long long)d->expert_begin,
                    (long long)d->expert_end, (long long)d->n_expert);
    const int64_t held = d->expert_end - d->expert_begin;
    int rc;
    if (d->router && (rc = check_dense(ctx, d->router, d->n_expert, d->n_embd, "router"))) return rc;
    if ((rc = check_experts(ctx, d->gate_exps, held, d->n_embd, d->n_ff, "gate_exps"))) return rc;
    if ((rc = check_experts(ctx, d->up_exps, held, d->n_embd, d->n_ff, "up_exps"))) return rc;
    if ((rc = check_experts(ctx, d->down_exps, held, d->n_ff, d->n_embd, "down_exps"))) return rc;
    if (d->gate_exps->quant != d->up_exps->quant)
        return fail(ctx, STRATA_ERR_UNSUPPORTED_QUANT, "moe: gate_exps and up_exps must share a quant type");
    if (d->gate_shexp) {
        if (d->n_ff_shexp <= 0) return fail(ctx, STRATA_ERR_INVALID, "moe: n_ff_shexp %lld", (long long)d->n_ff_shexp);
        if ((rc = check_dense(ctx, d->gate_shexp, d->n_ff_shexp, d->n_embd, "gate_shexp"))) return rc;
        if ((rc = check_dense(ctx, d->up_shexp, d->n_ff_shexp, d->n_embd, "up_shexp"))) return rc;
        if ((rc = check_dense(ctx, d->down_shexp, d->n_embd, d->n_ff_shexp, "down_shexp"))) return rc;
        if ((rc = check_dense(ctx, d->gate_inp_shexp, 1, d->n_embd, "gate_inp_shexp"))) return rc;
    }
    if (!ctx->aux) {  // the shared expert's stream; without it the layer runs in line
        cudaSetDevice(ctx->device);
        // decode (one or two tokens): the highest priority, so the shared
        // expert's small grids take SM slots as the routed passes' CTAs retire
        // instead of queueing behind them; otherwise the default priority
        int lo_pri = 0, hi_pri = 0;
        cudaDeviceGetStreamPriorityRange(&lo_pri, &hi_pri);
        if (cudaStreamCreateWithPriority(&ctx->aux, cudaStreamNonBlocking, hi_pri) != cudaSuccess ||
            cudaStreamCreateWithFlags(&ctx->aux_lo, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&ctx->fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ctx->join, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            if (ctx->fork) cudaEventDestroy(ctx->fork);
            if (ctx->join) cudaEventDestroy(ctx->join);
            if (ctx->aux) cudaStreamDestroy(ctx->aux);
            if (ctx->aux_lo) cudaStreamDestroy(ctx->aux_lo);
            ctx->aux = ctx->aux_lo = nullptr;
            ctx->fork = ctx->join = nullptr;
        }
    }
    strata_moe* L = new strata_moe();
    L->ctx = ctx;
    L->d = *d;
    ctx->moes.insert(L);
    *out = L;
    return STRATA_OK;
}

int strata_cuda_moe_destroy(strata_moe* L) {
    if (!L || L->magic != kMoeMagic) return STRATA_ERR_INVALID;
    L->magic = 0;
    if (L->ctx) {  // null once its context was destroyed (the graphs went with it)
        std::lock_guard<std::mutex> g(L->ctx->mu);
        cudaSetDevice(L->ctx->device);
        release_graphs(L);
        L->ctx->moes.erase(L);
    }
    delete L;
    return STRATA_OK;
}

int strata_cuda_moe_ffn_dev(strata_ctx* ctx, const strata_moe* L, const float* x, const float* logits, int64_t T,
                            float* out, int32_t* ids, float* wts, void* stream) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_moe(ctx, L);
    if (rc) return rc;
    if (!x || !out) return fail(ctx, STRATA_ERR_INVALID, "moe: null x or out");
    cudaSetDevice(ctx->device);
    return moe_enqueue(ctx, L, x, logits, T, out, ids, wts, pick_stream(ctx, stream));
}

int strata_cuda_moe_ffn(strata_ctx* ctx, const strata_moe* L, const float* x, const float* logits, int64_t T,
                        float* out, int32_t* ids, float* wts) {
    if (!ctx) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = check_moe(ctx, L);
    if (rc) return rc;
    if (!x || !out) return fail(ctx, STRATA_ERR_INVALID, "moe: null x or out");
    if (T < 1) return fail(ctx, STRATA_ERR_INVALID, "moe: tokens %lld", (long long)T);
    cudaSetDevice(ctx->device);
    const strata_moe_desc& d = L->d;
    const size_t xb = (size_t)T * (size_t)d.n_embd * 4, lb = logits ? (size_t)T * (size_t)d.n_expert * 4 : 0;
    const size_t rb = (size_t)T * (size_t)d.top_k * 4;
    const size_t in_bytes = xb + ((lb + 255) & ~size_t(255));
    const size_t out_bytes = xb + 2 * ((rb + 255) & ~size_t(255));
    if ((rc = ensure_device(ctx, ctx->x_dev, in_bytes + 256, "cudaMalloc(x)"))) return rc;
    if ((rc = ensure_device(ctx, ctx->y_dev, out_bytes + 512, "cudaMalloc(out)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->x_host, in_bytes + 256, "cudaMallocHost(x)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->y_host, out_bytes + 512, "cudaMallocHost(out)"))) return rc;
    uint8_t* hx = static_cast<uint8_t*>(ctx->x_host.ptr);
    uint8_t* dx = static_cast<uint8_t*>(ctx->x_dev.ptr);
    uint8_t* dy = static_cast<uint8_t*>(ctx->y_dev.ptr);
    uint8_t* hy = static_cast<uint8_t*>(ctx->y_host.ptr);
    const size_t lo = (xb + 255) & ~size_t(255);
    const size_t io = (xb + 255) & ~size_t(255), wo = io + ((rb + 255) & ~size_t(255));
    memcpy(hx, x, xb);
    if (logits) memcpy(hx + lo, logits, lb);
    // input copy, the layer, output copy: all on the context stream (the
    // shared expert forks from it and joins back)
    auto enqueue = [&]() -> int {
        cudaError_t e = cudaMemcpyAsync(dx, hx, lo + lb, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(H2D)");
        int r = moe_enqueue(ctx, L, reinterpret_cast<const float*>(dx),
                            logits ? reinterpret_cast<const float*>(dx + lo) : nullptr, T, reinterpret_cast<float*>(dy),
                            reinterpret_cast<int32_t*>(dy + io), reinterpret_cast<float*>(dy + wo), ctx->stream);
        if (r) return r;
        e = cudaMemcpyAsync(hy, dy, wo + rb, cudaMemcpyDeviceToHost, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(D2H)");
        return STRATA_OK;
    };
    // A token count seen before with the same buffers replays its graph: one
    // launch instead of the chain's dozen, so the device never waits for the
    // host between kernels. The first call of a count runs directly (it sizes
    // the buffers) and then captures the graph for the next one.
    MoeGraph* hit = nullptr;
    for (MoeGraph& m : L->graphs)
        if (m.exec && m.T == T && m.logits == (logits != nullptr) && m.gen == ctx->buf_gen) hit = &m;
    if (hit) {
        hit->used = ++L->tick;
        cudaError_t e = cudaGraphLaunch(hit->exec, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGraphLaunch(moe layer)");
    } else if ((rc = enqueue())) {
        return rc;
    }
    if ((rc = wait_stream(ctx, ctx->stream))) return rc;
    if (!hit) capture_layer(ctx, L, T, logits != nullptr, enqueue);
    memcpy(out, hy, xb);
    if (ids) memcpy(ids, hy + io, rb);
    if (wts) memcpy(wts, hy + wo, rb);
    return STRATA_OK;
}

}  // extern "C"
