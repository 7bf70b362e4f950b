/*
 * strata_cuda.h — C ABI of the B200 quantized-matmul backend for strata-rs.
 *
 * This is the boundary a `strata-backend-cuda` crate binds (`extern "C"`):
 * plain pointers and sizes, no torch or CUDA types in any signature. Every
 * function returns a status (STRATA_OK = 0); the message of the last failure
 * on a context is strata_cuda_last_error(ctx).
 *
 * Reference interface being replaced (paths relative to the strata-rs repo):
 *   trait ComputeBackend ............. crates/strata-core/src/backend.rs:20-51
 *   ComputeBackend::gemv ............. crates/strata-core/src/backend.rs:25
 *   ComputeBackend::expert_gemv ...... crates/strata-core/src/backend.rs:28-35
 *   QuantTensor (rows = OUT) ......... crates/strata-core/src/backend.rs:114-154
 *   ExpertView ([E][IN][OUT]) ........ crates/strata-core/src/weights.rs:11-34
 *   dequantize_row ................... crates/strata-gguf/src/dequant.rs:45-61
 *   MoeLayer::route / combine ........ crates/strata-core/src/moe.rs:48-144
 *   Error::Backend { message } ....... crates/strata-core/src/error.rs:31-32
 *
 * Threading: a context may be shared between threads (the trait is
 * Send + Sync); calls on one context are serialised by an internal mutex.
 * Host-buffer calls are synchronous: results are in the output buffer when
 * the call returns, as the trait requires. The *_dev variants take device
 * pointers and only enqueue work on the given stream (NULL = the context's
 * own stream).
 */
#ifndef STRATA_CUDA_H
#define STRATA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define STRATA_CUDA_ABI_VERSION 1

/* Status codes. STRATA_ERR_UNSUPPORTED_QUANT and STRATA_ERR_TRUNCATED are the
 * two strata_gguf::Error variants dequantize_row returns
 * (crates/strata-gguf/src/dequant.rs:50-55, :102-105); everything else maps
 * to strata_core::Error::Backend. */
enum {
    STRATA_OK = 0,
    STRATA_ERR_INVALID = 1,           /* bad argument, shape or handle */
    STRATA_ERR_UNSUPPORTED_QUANT = 2, /* quant type not on this path */
    STRATA_ERR_TRUNCATED = 3,         /* byte slice shorter than the shape needs */
    STRATA_ERR_CUDA = 4,              /* a CUDA runtime call failed */
    STRATA_ERR_OOM = 5,               /* device allocation failed */
    STRATA_ERR_TIMEOUT = 6,           /* a bounded wait on the device expired */
    STRATA_ERR_NCCL = 7,              /* a collective failed */
    STRATA_ERR_BUDGET = 8,            /* the weight budget would be exceeded */
    STRATA_ERR_SCRATCH_LIMIT = 9      /* too large for strata_cuda_gemv_noalloc's fixed scratch */
};

/* Strata ggml type ids accepted here (crates/strata-gguf/src/quant.rs:15-43). */
enum {
    STRATA_QUANT_F32 = 0,
    STRATA_QUANT_F16 = 1,
    STRATA_QUANT_Q8_0 = 8,
    STRATA_QUANT_Q4_K = 12,
    STRATA_QUANT_Q5_K = 13,
    STRATA_QUANT_Q6_K = 14,
    STRATA_QUANT_BF16 = 30
};

typedef struct strata_ctx strata_ctx;       /* one device, one stream */
typedef struct strata_weight strata_weight; /* a tensor resident in HBM */

/* ---------------------------------------------------------------- context */

int strata_cuda_abi_version(void);

/* ComputeBackend::name (backend.rs:22): always "cuda". */
const char *strata_cuda_name(void);

/* Creates a context on `device` (its own non-blocking stream, pinned staging). */
int strata_cuda_create(int device, strata_ctx **out);
/* Waits (bounded) for the context's work, then frees everything it owns:
 * buffers, streams, the communicator, and any weight not yet released with
 * strata_cuda_free_weight (those handles become invalid). MoE layers built
 * on its weights must not be used afterwards. */
int strata_cuda_destroy(strata_ctx *ctx);

/* Message of the last failure on ctx ("" if none). Valid until the next call. */
const char *strata_cuda_last_error(const strata_ctx *ctx);

/* Caps the HBM bytes weights may occupy (0 = no cap). The CLI's
 * --gpu-weights-mib (crates/strata-cli/src/main.rs:116-118) maps here. */
int strata_cuda_set_weight_budget(strata_ctx *ctx, uint64_t bytes);
int strata_cuda_resident_bytes(const strata_ctx *ctx, uint64_t *out);

/* Bound, in milliseconds, on every host wait for device work (default 60000).
 * An expired wait returns STRATA_ERR_TIMEOUT and leaves the context usable. */
int strata_cuda_set_wait_timeout_ms(strata_ctx *ctx, uint32_t ms);

/* Which kernels serve the decode GEMV: AUTO picks the tensor-core kernel for
 * Q4_K / Q5_K and the CUDA-core kernels otherwise; the others force one family
 * (TENSOR_CORES fails with STRATA_ERR_UNSUPPORTED_QUANT where it has no kernel).
 * Both families meet the same tolerance; the switch exists for diagnosis. */
enum { STRATA_GEMV_AUTO = 0, STRATA_GEMV_CUDA_CORES = 1, STRATA_GEMV_TENSOR_CORES = 2 };
int strata_cuda_set_gemv_path(strata_ctx *ctx, int path);

/* Waits (bounded) for all work enqueued on the context's stream. */
int strata_cuda_synchronize(strata_ctx *ctx);

/* The context's stream as an opaque cudaStream_t. */
int strata_cuda_stream(const strata_ctx *ctx, void **stream_out);

/* ---------------------------------------------------------------- weights */

/* Copies a tensor's bytes to HBM unchanged (the strata-gguf payload slice,
 * GgufFile::tensor_data, crates/strata-gguf/src/reader.rs:425-445).
 *   dense   (QuantTensor): n_expert = 0, rows = OUT, cols = IN
 *   experts (ExpertView):  n_expert = E, rows = IN,  cols = OUT
 * Each row is quantized along `cols`. `len` must cover
 * max(1, n_expert) * rows * byte_size(cols); cols must be a whole number of
 * blocks (else STRATA_ERR_TRUNCATED, as dequantize_row). */
int strata_cuda_upload(strata_ctx *ctx, const uint8_t *bytes, size_t len, uint32_t quant,
                       int64_t n_expert, int64_t rows, int64_t cols, strata_weight **out);
int strata_cuda_free_weight(strata_weight *w);

/* Many tensors in one pass (a model load: WeightStore::new,
 * crates/strata-core/src/weights.rs:49-67, walking every shard's tensors).
 * Each item means what strata_cuda_upload's arguments mean. The bytes of all
 * items stream through the same two pinned chunks, so the host threads that
 * fill one chunk take the next tensor's page faults while the DMA engine
 * drains the other. All or nothing: on an error no item stays resident and
 * every out[i] is NULL; the message names the failing item. */
typedef struct {
    const uint8_t *bytes;
    size_t len;
    uint32_t quant;
    int64_t n_expert, rows, cols;
} strata_upload;
int strata_cuda_upload_many(strata_ctx *ctx, const strata_upload *items, int64_t n,
                            strata_weight **out);

/* Dequantizes rows [row0, row0 + nrows) of expert `expert` (0 for dense)
 * into out_host (nrows * cols f32). Bit-exact with dequantize_row. */
int strata_cuda_dequant(strata_ctx *ctx, const strata_weight *w, int64_t expert, int64_t row0,
                        int64_t nrows, float *out_host);

/* ------------------------------------------------------------ decode GEMV */

/* ComputeBackend::gemv (backend.rs:25) over `batch` (1..8) activation rows:
 * x is batch x cols f32, y is batch x rows f32 (row-major). The _dev variant
 * needs x 16-byte aligned; its first call may size the context's workspace
 * (a device allocation), so make one call before capturing it in a graph.
 * The workspace is per context: _dev calls of one context on different
 * streams must not overlap. */
int strata_cuda_gemv(strata_ctx *ctx, const strata_weight *w, const float *x, float *y, int batch);
int strata_cuda_gemv_dev(strata_ctx *ctx, const strata_weight *w, const float *x_dev, float *y_dev,
                         int batch, void *stream);

/* ComputeBackend::expert_gemv (backend.rs:28-35) for expert e:
 * x is batch x rows(IN), y is batch x cols(OUT). */
int strata_cuda_expert_gemv(strata_ctx *ctx, const strata_weight *w, int64_t e, const float *x,
                            float *y, int batch);
int strata_cuda_expert_gemv_dev(strata_ctx *ctx, const strata_weight *w, int64_t e,
                                const float *x_dev, float *y_dev, int batch, void *stream);

/* ------------------------------------------------------------ prefill GEMM */

/* The prompt-prefill form of ComputeBackend::gemv: the reference runs one
 * gemv per prompt token (crates/strata-core/src/generate.rs:116-118, through
 * ops::gemv, crates/strata-core/src/ops.rs:14-28); this computes all m tokens
 * at once on the tensor cores. y (m x rows f32) = x (m x cols) W^T for a dense
 * Q4_K, Q5_K or Q6_K tensor whose cols is a multiple of 256 and whose row size
 * in bytes is a multiple of 16. Activations are staged as bf16: the _bf16
 * entry points take bf16 bit patterns, the _f32 ones round f32 to bf16
 * (nearest even) on the device first; outputs match gemv on the bf16-rounded
 * activations within relative error 1e-2. Other quant types return
 * STRATA_ERR_UNSUPPORTED_QUANT (use strata_cuda_gemv per token). The _dev
 * variants need x 16-byte aligned and may size the context's workspace on
 * their first call for a shape; workspace rules as for strata_cuda_gemv_dev. */
int strata_cuda_gemm_bf16(strata_ctx *ctx, const strata_weight *w, const uint16_t *x, float *y, int64_t m);
int strata_cuda_gemm_bf16_dev(strata_ctx *ctx, const strata_weight *w, const uint16_t *x_dev,
                              float *y_dev, int64_t m, void *stream);
int strata_cuda_gemm_f32(strata_ctx *ctx, const strata_weight *w, const float *x, float *y, int64_t m);
int strata_cuda_gemm_f32_dev(strata_ctx *ctx, const strata_weight *w, const float *x_dev, float *y_dev,
                             int64_t m, void *stream);

/* Weight staging of the GEMM: 2 (default) = bf16 hi + bf16 residual, the
 * precision the 1e-2 bound needs; 1 = a single bf16 copy, about half the
 * tensor work but outside that bound (kept for measurement only). */
int strata_cuda_set_gemm_terms(strata_ctx *ctx, int terms);

/* ---------------------------------------------------------------- MoE layer */

/* One MoE layer resident on the device: the weights of strata_core::moe::MoeLayer
 * (crates/strata-core/src/moe.rs:22-35) as uploaded handles. Expert tensors
 * are uploaded with n_expert = the number of experts this context holds:
 * all of them on one GPU, the slice [expert_begin, expert_end) under expert
 * parallelism (ids stay global). The shared expert is optional (NULL
 * gate_shexp) and runs only where with_shared is set. */
typedef struct strata_moe strata_moe;
typedef struct {
    const strata_weight *router;          /* [n_expert rows][n_embd]; may be NULL when logits are given */
    const strata_weight *gate_exps;       /* experts [held][n_embd][n_ff] */
    const strata_weight *up_exps;         /* experts [held][n_embd][n_ff] */
    const strata_weight *down_exps;       /* experts [held][n_ff][n_embd] */
    const strata_weight *gate_shexp;      /* [n_ff_shexp][n_embd] or NULL */
    const strata_weight *up_shexp;        /* [n_ff_shexp][n_embd] */
    const strata_weight *down_shexp;      /* [n_embd][n_ff_shexp] */
    const strata_weight *gate_inp_shexp;  /* [1][n_embd] */
    int64_t n_embd, n_expert, top_k, n_ff, n_ff_shexp;
    int64_t expert_begin, expert_end;     /* experts held here: [begin, end) */
    int with_shared;                      /* run the shared expert in this context */
} strata_moe_desc;

/* Validates shapes and quant types (experts: Q4_K, Q5_K, Q6_K or Q8_0 with
 * n_ff and n_embd multiples of 256; n_expert <= 1024; top_k <= 32). The
 * handles must outlive the layer. */
int strata_cuda_moe_create(strata_ctx *ctx, const strata_moe_desc *desc, strata_moe **out);
int strata_cuda_moe_destroy(strata_moe *layer);

/* MoeLayer::route + MoeLayer::combine (moe.rs:48-144) for `tokens` tokens:
 * x and out are tokens x n_embd f32. Routing comes from router_logits
 * (tokens x n_expert f32) when given, else from the router GEMV on the
 * bf16-rounded x (moe.rs:55-56). Under expert parallelism `out` holds this
 * context's partial sum (its experts, plus the shared expert where held);
 * the sum over contexts is the layer output. ids_out / weights_out
 * (tokens x top_k, optional) receive the routing: global expert ids in
 * ascending order and their renormalised weights. */
int strata_cuda_moe_ffn(strata_ctx *ctx, const strata_moe *layer, const float *x, const float *router_logits,
                        int64_t tokens, float *out, int32_t *ids_out, float *weights_out);
int strata_cuda_moe_ffn_dev(strata_ctx *ctx, const strata_moe *layer, const float *x_dev,
                            const float *router_logits_dev, int64_t tokens, float *out_dev,
                            int32_t *ids_dev, float *weights_dev, void *stream);

/* ------------------------------------------------------- elementwise trait ops */

/* ComputeBackend's elementwise methods (crates/strata-core/src/backend.rs:37-50),
 * with CpuBackend's arithmetic (crates/strata-backend-cpu/src/lib.rs:44-67,
 * crates/strata-core/src/ops.rs): f64 sums and products where ops.rs uses f64,
 * the f32 exp of softmax as the f64 exp rounded to f32. The host forms take
 * one slice per call, as the trait does (synchronous, host buffers); the
 * device forms take `rows` (or `heads`) vectors at once on `stream`, so a
 * layer's activations can stay in device memory.
 *   rms_norm   x = x * w / sqrt(mean(x^2) + eps)          ops.rs:45-56
 *   l2_norm    x = x / sqrt(sum(x^2) + eps)               ops.rs:71-81
 *   softmax    max-shifted, f64 sum                       ops.rs:107-119
 *   rope_neox  NEOX pairs (i, i + n_rot/2) of the first min(n_rot, head_dim,
 *              len) & ~1 dims, angle = freq_base^(-2i/n_rot') * pos  ops.rs:121-140
 *   add        a += b                                     ops.rs:164-168 */
int strata_cuda_rms_norm(strata_ctx *ctx, float *x, const float *w, int64_t n, double eps);
int strata_cuda_l2_norm(strata_ctx *ctx, float *head, int64_t n, double eps);
int strata_cuda_softmax(strata_ctx *ctx, float *xs, int64_t n);
int strata_cuda_rope_neox(strata_ctx *ctx, float *head, int64_t len, int64_t pos, int64_t n_rot, int64_t head_dim,
                          double freq_base);
int strata_cuda_add(strata_ctx *ctx, float *a, const float *b, int64_t n);
int strata_cuda_rms_norm_dev(strata_ctx *ctx, float *x_dev, const float *w_dev, int64_t n, int64_t rows, double eps,
                             void *stream);
int strata_cuda_l2_norm_dev(strata_ctx *ctx, float *x_dev, int64_t head_dim, int64_t heads, double eps,
                            void *stream);
int strata_cuda_softmax_dev(strata_ctx *ctx, float *x_dev, int64_t n, int64_t rows, void *stream);
int strata_cuda_rope_neox_dev(strata_ctx *ctx, float *x_dev, int64_t head_dim, int64_t heads, int64_t n_rot,
                              int64_t pos, double freq_base, void *stream);
int strata_cuda_add_dev(strata_ctx *ctx, float *a_dev, const float *b_dev, int64_t n, void *stream);

/* ------------------------------------------------------------------ multi-GPU */

/* No counterpart in the reference, which runs on one device: the sharded
 * forms of its gemv and MoE layer, one process (and one context) per GPU.
 * strata_cuda_comm_unique_id is called on one rank; its bytes reach the other
 * ranks by the caller's means (e.g. a torch.distributed broadcast), then every
 * rank calls strata_cuda_comm_init. Init waits at most the context's wait
 * timeout for the other ranks (STRATA_ERR_TIMEOUT), so a rank that never
 * joins does not block the others forever. */
#define STRATA_COMM_ID_BYTES 128
int strata_cuda_comm_unique_id(uint8_t *id_out /* STRATA_COMM_ID_BYTES */);
int strata_cuda_comm_init(strata_ctx *ctx, int rank, int world, const uint8_t *id);
int strata_cuda_comm_info(const strata_ctx *ctx, int *rank, int *world);

/* Collectives issued between group_start and group_end (the gathers of
 * several sharded GEMV calls, MoE all-reduces) are launched together at
 * group_end, as one NCCL group: one collective launch for a whole decode step.
 * The GEMV and MoE calls enqueue their own kernels at once; only their
 * collectives wait for group_end. The sharded GEMM cannot run inside a group
 * (its transpose follows its gather). Groups nest. */
int strata_cuda_comm_group_start(strata_ctx *ctx);
int strata_cuda_comm_group_end(strata_ctx *ctx);

/* Row-sharded projection: w holds this rank's rows [rank R, (rank + 1) R) of
 * an OUT = world * R row matrix (every rank the same R). The local GEMV
 * (batch 1..8) or prefill GEMM (m tokens, bf16 x) writes its slice and an
 * all-gather over NVLink fills y_dev (batch | m) x OUT on every rank. */
int strata_cuda_gemv_sharded_dev(strata_ctx *ctx, const strata_weight *w_shard, const float *x_dev, float *y_dev,
                                 int batch, void *stream);
int strata_cuda_gemm_sharded_dev(strata_ctx *ctx, const strata_weight *w_shard, const uint16_t *x_dev,
                                 float *y_dev, int64_t m, void *stream);

/* How the sharded GEMV gathers its rows. PEER runs the all-gather over peer
 * memory with no NCCL call: the tensor-core GEMV writes its columns into this
 * rank's exchange buffer (device memory that every rank mapped with CUDA IPC
 * at comm_init), then one all-gather kernel pushes them into every other
 * rank's buffer over NVLink (16-byte stores), signals the other ranks, waits
 * for their signals (bounded by the context's wait timeout, then
 * STRATA_ERR_TIMEOUT) and assembles y. Inside a collective group that kernel
 * runs once, at group_end, for all the group's calls on one stream (y is
 * complete after group_end's work, as with NCCL). The calls are
 * graph-capturable. NCCL uses the per-row in-place all-gathers. AUTO (the
 * default) takes PEER where it applies -- peer memory available on every
 * rank, a Q4_K / Q5_K shard on the tensor-core path with a multiple of 4 rows,
 * y 16-byte aligned, batch x OUT within the exchange capacity -- and NCCL
 * otherwise. The mode also picks the expert-parallel MoE layer's all-reduce:
 * PEER sums the ranks' partial outputs over the same exchange buffers (every
 * rank adds the G partials in rank order, so all ranks get the same bits),
 * NCCL calls ncclAllReduce. Every rank must set the same mode (the ranks of
 * one call must take the same path). */
enum { STRATA_GATHER_AUTO = 0, STRATA_GATHER_NCCL = 1, STRATA_GATHER_PEER = 2 };
int strata_cuda_comm_set_gather(strata_ctx *ctx, int mode);
/* available: 1 if every rank opened every peer's exchange buffer;
 * capacity_floats: the largest batch x OUT the PEER path gathers. */
int strata_cuda_comm_peer_info(const strata_ctx *ctx, int *available, int64_t *capacity_floats);

/* Expert-parallel MoE layer: this rank's partial sum (its experts, plus the
 * shared expert on the rank whose layer has with_shared) all-reduced, so
 * out_dev holds the full layer output on every rank. */
int strata_cuda_moe_ffn_ep_dev(strata_ctx *ctx, const strata_moe *layer, const float *x_dev,
                               const float *router_logits_dev, int64_t tokens, float *out_dev, void *stream);

/* ------------------------------------------------- decode GEMV, no allocation */

/* No counterpart in the reference: an addition for callers that must not
 * allocate device memory -- code running while a stream is being captured into
 * a CUDA graph (where a cudaMalloc would break the capture), engines whose
 * device memory all comes from their own pre-sized pool, or hosts where
 * another runtime owns the allocator. It needs no context.
 *
 * The same tensor-core decode GEMV as strata_cuda_gemv_dev: y = W x for a
 * Q4_K or Q5_K matrix already in device memory in strata-gguf's byte layout
 * (w_dev, 16-byte aligned; rows = OUT, cols = IN, a multiple of 256), x
 * batch x cols f32 and y batch x rows f32 on the device, work enqueued on
 * `stream` (NULL = the legacy default stream). Its scratch is a 320 KiB
 * static device array inside this library, so it allocates nothing; the
 * limit is cols * batch <= 65,536 (e.g. K = 8192 at batch 8), beyond which it
 * returns STRATA_ERR_SCRATCH_LIMIT without launching.
 *
 * The first call on a device looks up the array's device address (with that
 * device current), so make one call on each device before capturing a stream.
 * Every call shares the one array: calls that can overlap on the GPU (other
 * streams, other threads) race on it and must be serialised by the caller.
 * The scratch keeps the last call's contents; each call rewrites all of it
 * that it reads. Returns without synchronising; a kernel whose bounded wait
 * expired is reported by strata_cuda_gemv_noalloc_status. An error already
 * pending from earlier work makes the call return STRATA_ERR_CUDA unlaunched. */
int strata_cuda_gemv_noalloc(const uint8_t *w_dev, uint32_t quant, int64_t rows, int64_t cols,
                             const float *x_dev, float *y_dev, int batch, void *stream);

/* No counterpart in the reference: the status of strata_cuda_gemv_noalloc on
 * the current device after the work queued on `stream` (it waits for that
 * stream). STRATA_ERR_TIMEOUT if any of its kernels since the last clear gave
 * up a bounded wait (that call's y is incomplete), else STRATA_OK. With
 * `clear` non-zero the recorded timeout is reset. Allocates nothing (one word
 * is copied to the host and, when clearing, back). */
int strata_cuda_gemv_noalloc_status(void *stream, int clear);

#ifdef __cplusplus
}
#endif
#endif /* STRATA_CUDA_H */
