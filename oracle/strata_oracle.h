/*
 * strata_oracle.h — CPU restatement of strata-rs's quantized-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the CUDA path is
 * compared against; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it. The product (libstrata_cuda.so) never links or
 * calls it.
 *
 * Every function restates one function of the reference (paths relative to
 * the strata-rs repository root) in plain C11, compiled with
 * -O2 -ffp-contract=off so that `a * b - c` rounds twice, as Rust does.
 */
#ifndef STRATA_ORACLE_H
#define STRATA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Strata ggml type ids: crates/strata-gguf/src/quant.rs:15-43 */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6, ORC_Q5_1 = 7,
    ORC_Q8_0 = 8, ORC_Q8_1 = 9, ORC_Q2_K = 10, ORC_Q3_K = 11, ORC_Q4_K = 12, ORC_Q5_K = 13,
    ORC_Q6_K = 14, ORC_IQ4_NL = 20, ORC_IQ4_XS = 23, ORC_BF16 = 30, ORC_MXFP4 = 39,
    ORC_NVFP4 = 40, ORC_Q2_0 = 42
};

/* status codes (mirrors strata_core::Error's variants used on this path) */
enum { ORC_OK = 0, ORC_ERR_UNSUPPORTED = 2, ORC_ERR_TRUNCATED = 3, ORC_ERR_INVALID = 1 };

/* QuantType::block_size / type_size / byte_size: quant.rs:125-180.
 * Return 0 for an id this path does not cover. */
int64_t orc_block_size(uint32_t quant);
int64_t orc_type_size(uint32_t quant);
int64_t orc_byte_size(uint32_t quant, int64_t n_elements);

/* half 2.7.1 f16::from_bits(h).to_f32(): crates/strata-gguf/src/dequant.rs:33-36 */
float orc_f16_to_f32(uint16_t h);
/* half 2.7.1 bf16::from_f32(v).to_f32(): crates/strata-core/src/hyper.rs:21-24 */
float orc_bf16_round(float v);
uint16_t orc_f32_to_bf16_bits(float v);

/* dequantize_row: crates/strata-gguf/src/dequant.rs:45-61 (+ per-type blocks) */
int orc_dequantize_row(uint32_t quant, const uint8_t *block, size_t block_len,
                       float *out, int64_t n);

/* ops::gemv: crates/strata-core/src/ops.rs:14-28. W is rows x cols (rows = OUT). */
int orc_gemv(uint32_t quant, const uint8_t *w, size_t w_len, int64_t rows, int64_t cols,
             const float *x, float *y);
/* The same product over `batch` activation columns (x: batch x cols, y: batch x rows),
 * one ops::gemv per column; threads > 1 splits rows across pthreads (the
 * row-parallel restatement of the README's rayon claim). */
int orc_gemv_batch(uint32_t quant, const uint8_t *w, size_t w_len, int64_t rows, int64_t cols,
                   const float *x, float *y, int64_t batch, int threads);
/* One activation column, output rows [row0, row_end) only: y holds row_end-row0
 * values. Used for bounded CPU-baseline samples of a large matrix. */
int orc_gemv_rows(uint32_t quant, const uint8_t *w, size_t w_len, int64_t rows, int64_t cols,
                  const float *x, float *y, int64_t row0, int64_t row_end, int threads);

/* ops::expert_gemv: crates/strata-core/src/ops.rs:169-195.
 * W: n_expert x rows(IN) x cols(OUT), each row quantized along cols. */
int orc_expert_gemv(uint32_t quant, const uint8_t *w, size_t w_len, int64_t n_expert,
                    int64_t rows, int64_t cols, int64_t e, const float *x, float *y);

/* ops::silu / ops::sigmoid: crates/strata-core/src/ops.rs:84-92 */
float orc_silu(float x);
float orc_sigmoid(float x);

/* The elementwise trait methods of ComputeBackend (crates/strata-core/src/backend.rs:37-50)
 * as CpuBackend runs them (crates/strata-backend-cpu/src/lib.rs:44-67), one vector per call:
 *   ops::rms_norm   crates/strata-core/src/ops.rs:45-56  f64 sum of squares / n, x*scale*w
 *   ops::l2_norm    crates/strata-core/src/ops.rs:71-81  f64 sum of squares, x*inv
 *   ops::softmax    crates/strata-core/src/ops.rs:107-119 max shift, f32 exp, f64 sum
 *   ops::rope_neox  crates/strata-core/src/ops.rs:121-140 NEOX pairs (i, i + n_rot/2), f64 angles
 *   ops::add_into   crates/strata-core/src/ops.rs:164-168 out += a in f32 */
void orc_rms_norm(float *x, const float *w, int64_t n, double eps);
void orc_l2_norm(float *head, int64_t n, double eps);
void orc_softmax(float *xs, int64_t n);
void orc_rope_neox(float *head, int64_t len, int64_t pos, int64_t n_rot, int64_t head_dim, double freq_base);
void orc_add(float *out, const float *a, int64_t n);

/* test support: inputs where the C library's expf is not correctly rounded */
int64_t orc_expf_misrounded(float lo, float hi, float *out, int64_t cap);
int64_t orc_expf_tie_pairs(float lo, float hi, float *out, int64_t cap);

/* MoeLayer::route from the router logits on (crates/strata-core/src/moe.rs:57-91):
 * softmax (max-shift, f64 sum, f32 inv), stable top-k, ids ascending,
 * renormalised with a 2^-14 floor. logits is overwritten with the probs. */
int orc_moe_route_logits(float *logits, int64_t n_expert, int64_t top_k,
                         int64_t *ids_out, float *weights_out);

/* One MoE layer's weights, as strata_core::moe::MoeLayer holds them. */
typedef struct {
    uint32_t quant_router;  const uint8_t *router;  size_t router_len;   /* [n_expert, n_embd] */
    uint32_t quant_gate_exps; const uint8_t *gate_exps; size_t gate_exps_len; /* [E][n_embd][n_ff] */
    uint32_t quant_up_exps;   const uint8_t *up_exps;   size_t up_exps_len;
    uint32_t quant_down_exps; const uint8_t *down_exps; size_t down_exps_len; /* [E][n_ff][n_embd] */
    uint32_t quant_gate_shexp; const uint8_t *gate_shexp; size_t gate_shexp_len; /* [n_ff_sh, n_embd] */
    uint32_t quant_up_shexp;   const uint8_t *up_shexp;   size_t up_shexp_len;
    uint32_t quant_down_shexp; const uint8_t *down_shexp; size_t down_shexp_len; /* [n_embd, n_ff_sh] */
    uint32_t quant_gate_inp_shexp; const uint8_t *gate_inp_shexp; size_t gate_inp_shexp_len; /* [1, n_embd] */
    int64_t n_embd, n_expert, top_k, n_ff, n_ff_shexp;
} orc_moe_weights;

/* MoeLayer::route with the router gemv on the bf16-rounded input (moe.rs:48-92). */
int orc_moe_route(const orc_moe_weights *L, const float *x, int64_t *ids_out, float *weights_out);

/* MoeLayer::combine (moe.rs:97-144) for one token, given its routing. */
int orc_moe_combine(const orc_moe_weights *L, const float *x, const int64_t *ids,
                    const float *weights, float *out);

/* The whole layer for `tokens` tokens: route (from `logits` [tokens, n_expert]
 * when non-NULL, else through the router) then combine; out is [tokens, n_embd].
 * threads > 1 splits tokens across pthreads. ids/weights (tokens x top_k) may be NULL. */
int orc_moe_layer(const orc_moe_weights *L, const float *x, const float *logits, int64_t tokens,
                  float *out, int64_t *ids_out, float *weights_out, int threads);

#ifdef __cplusplus
}
#endif
#endif
