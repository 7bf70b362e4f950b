//! Raw bindings to `libstrata_cuda.so`: one declaration per function of
//! `include/strata_cuda.h` and `include/strata_gguf.h`, with the same names,
//! argument order and integer widths (a test of the C library checks the two
//! against each other).

#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

/// One device and its stream (`strata_ctx`).
#[repr(C)]
#[derive(Debug)]
pub(crate) struct StrataCtx {
    _p: [u8; 0],
}

/// A tensor resident in HBM (`strata_weight`).
#[repr(C)]
#[derive(Debug)]
pub(crate) struct StrataWeight {
    _p: [u8; 0],
}

/// A device MoE layer (`strata_moe`).
#[repr(C)]
#[derive(Debug)]
pub(crate) struct StrataMoe {
    _p: [u8; 0],
}

/// An opened GGUF model, every shard (`strata_gguf`).
#[repr(C)]
#[derive(Debug)]
pub(crate) struct StrataGguf {
    _p: [u8; 0],
}

pub(crate) const STRATA_CUDA_ABI_VERSION: c_int = 1;

pub(crate) const STRATA_OK: c_int = 0;
pub(crate) const STRATA_ERR_INVALID: c_int = 1;
pub(crate) const STRATA_ERR_UNSUPPORTED_QUANT: c_int = 2;
pub(crate) const STRATA_ERR_TRUNCATED: c_int = 3;
pub(crate) const STRATA_ERR_CUDA: c_int = 4;
pub(crate) const STRATA_ERR_OOM: c_int = 5;
pub(crate) const STRATA_ERR_TIMEOUT: c_int = 6;
pub(crate) const STRATA_ERR_NCCL: c_int = 7;
pub(crate) const STRATA_ERR_BUDGET: c_int = 8;
pub(crate) const STRATA_ERR_SCRATCH_LIMIT: c_int = 9;

pub(crate) const STRATA_ERR_IO: c_int = 10;
pub(crate) const STRATA_ERR_BAD_MAGIC: c_int = 11;
pub(crate) const STRATA_ERR_UNSUPPORTED_VERSION: c_int = 12;
pub(crate) const STRATA_ERR_BAD_VALUE_TYPE: c_int = 13;
pub(crate) const STRATA_ERR_BAD_KEY_LENGTH: c_int = 14;
pub(crate) const STRATA_ERR_STRING_NOT_UTF8: c_int = 15;
pub(crate) const STRATA_ERR_TENSOR_NOT_FOUND: c_int = 16;
pub(crate) const STRATA_ERR_WRONG_TENSOR_DIMS: c_int = 17;

pub(crate) const STRATA_GEMV_AUTO: c_int = 0;
pub(crate) const STRATA_GEMV_CUDA_CORES: c_int = 1;
pub(crate) const STRATA_GEMV_TENSOR_CORES: c_int = 2;

pub(crate) const STRATA_GATHER_AUTO: c_int = 0;
pub(crate) const STRATA_GATHER_NCCL: c_int = 1;
pub(crate) const STRATA_GATHER_PEER: c_int = 2;

pub(crate) const STRATA_COMM_ID_BYTES: usize = 128;

/// One tensor of a batched upload (`strata_upload`).
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct strata_upload {
    pub(crate) bytes: *const u8,
    pub(crate) len: usize,
    pub(crate) quant: u32,
    pub(crate) n_expert: i64,
    pub(crate) rows: i64,
    pub(crate) cols: i64,
}

/// The tensors and geometry of one MoE layer (`strata_moe_desc`).
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct strata_moe_desc {
    pub(crate) router: *const StrataWeight,
    pub(crate) gate_exps: *const StrataWeight,
    pub(crate) up_exps: *const StrataWeight,
    pub(crate) down_exps: *const StrataWeight,
    pub(crate) gate_shexp: *const StrataWeight,
    pub(crate) up_shexp: *const StrataWeight,
    pub(crate) down_shexp: *const StrataWeight,
    pub(crate) gate_inp_shexp: *const StrataWeight,
    pub(crate) n_embd: i64,
    pub(crate) n_expert: i64,
    pub(crate) top_k: i64,
    pub(crate) n_ff: i64,
    pub(crate) n_ff_shexp: i64,
    pub(crate) expert_begin: i64,
    pub(crate) expert_end: i64,
    pub(crate) with_shared: c_int,
}

/// One shard of an opened model (`strata_gguf_shard`).
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct strata_gguf_shard {
    pub(crate) path: *const c_char,
    pub(crate) version: u32,
    pub(crate) alignment: u64,
    pub(crate) data_start: u64,
    pub(crate) file_size: u64,
    pub(crate) n_tensors: i64,
    pub(crate) n_metadata: i64,
}

/// One tensor of the directory (`strata_gguf_tensor`).
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct strata_gguf_tensor {
    pub(crate) name: *const c_char,
    pub(crate) name_len: u64,
    pub(crate) type_: u32,
    pub(crate) n_dims: i32,
    pub(crate) dims: [u64; 4],
    pub(crate) offset: u64,
    pub(crate) shard: i32,
}

/// One metadata value (`strata_gguf_value`).
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub(crate) struct strata_gguf_value {
    pub(crate) type_: u32,
    pub(crate) i: i64,
    pub(crate) u: u64,
    pub(crate) f: f64,
    pub(crate) str_: *const c_char,
    pub(crate) str_len: u64,
    pub(crate) elem: u32,
    pub(crate) count: u64,
}

// include/strata_cuda.h
extern "C" {
    pub(crate) fn strata_cuda_abi_version() -> c_int;
    pub(crate) fn strata_cuda_name() -> *const c_char;
    pub(crate) fn strata_cuda_create(device: c_int, out: *mut *mut StrataCtx) -> c_int;
    pub(crate) fn strata_cuda_destroy(ctx: *mut StrataCtx) -> c_int;
    pub(crate) fn strata_cuda_last_error(ctx: *const StrataCtx) -> *const c_char;
    pub(crate) fn strata_cuda_set_weight_budget(ctx: *mut StrataCtx, bytes: u64) -> c_int;
    pub(crate) fn strata_cuda_resident_bytes(ctx: *const StrataCtx, out: *mut u64) -> c_int;
    pub(crate) fn strata_cuda_set_wait_timeout_ms(ctx: *mut StrataCtx, ms: u32) -> c_int;
    pub(crate) fn strata_cuda_set_gemv_path(ctx: *mut StrataCtx, path: c_int) -> c_int;
    pub(crate) fn strata_cuda_synchronize(ctx: *mut StrataCtx) -> c_int;
    pub(crate) fn strata_cuda_stream(ctx: *const StrataCtx, stream_out: *mut *mut c_void) -> c_int;
    pub(crate) fn strata_cuda_upload(
        ctx: *mut StrataCtx,
        bytes: *const u8,
        len: usize,
        quant: u32,
        n_expert: i64,
        rows: i64,
        cols: i64,
        out: *mut *mut StrataWeight,
    ) -> c_int;
    pub(crate) fn strata_cuda_free_weight(w: *mut StrataWeight) -> c_int;
    pub(crate) fn strata_cuda_upload_many(
        ctx: *mut StrataCtx,
        items: *const strata_upload,
        n: i64,
        out: *mut *mut StrataWeight,
    ) -> c_int;
    pub(crate) fn strata_cuda_dequant(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        expert: i64,
        row0: i64,
        nrows: i64,
        out_host: *mut f32,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemv(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        x: *const f32,
        y: *mut f32,
        batch: c_int,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemv_dev(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        x_dev: *const f32,
        y_dev: *mut f32,
        batch: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_expert_gemv(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        e: i64,
        x: *const f32,
        y: *mut f32,
        batch: c_int,
    ) -> c_int;
    pub(crate) fn strata_cuda_expert_gemv_dev(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        e: i64,
        x_dev: *const f32,
        y_dev: *mut f32,
        batch: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemm_bf16(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        x: *const u16,
        y: *mut f32,
        m: i64,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemm_bf16_dev(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        x_dev: *const u16,
        y_dev: *mut f32,
        m: i64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemm_f32(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        x: *const f32,
        y: *mut f32,
        m: i64,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemm_f32_dev(
        ctx: *mut StrataCtx,
        w: *const StrataWeight,
        x_dev: *const f32,
        y_dev: *mut f32,
        m: i64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_set_gemm_terms(ctx: *mut StrataCtx, terms: c_int) -> c_int;
    pub(crate) fn strata_cuda_moe_create(
        ctx: *mut StrataCtx,
        desc: *const strata_moe_desc,
        out: *mut *mut StrataMoe,
    ) -> c_int;
    pub(crate) fn strata_cuda_moe_destroy(layer: *mut StrataMoe) -> c_int;
    pub(crate) fn strata_cuda_moe_ffn(
        ctx: *mut StrataCtx,
        layer: *const StrataMoe,
        x: *const f32,
        router_logits: *const f32,
        tokens: i64,
        out: *mut f32,
        ids_out: *mut i32,
        weights_out: *mut f32,
    ) -> c_int;
    pub(crate) fn strata_cuda_moe_ffn_dev(
        ctx: *mut StrataCtx,
        layer: *const StrataMoe,
        x_dev: *const f32,
        router_logits_dev: *const f32,
        tokens: i64,
        out_dev: *mut f32,
        ids_dev: *mut i32,
        weights_dev: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_rms_norm(ctx: *mut StrataCtx, x: *mut f32, w: *const f32, n: i64, eps: f64) -> c_int;
    pub(crate) fn strata_cuda_l2_norm(ctx: *mut StrataCtx, head: *mut f32, n: i64, eps: f64) -> c_int;
    pub(crate) fn strata_cuda_softmax(ctx: *mut StrataCtx, xs: *mut f32, n: i64) -> c_int;
    pub(crate) fn strata_cuda_rope_neox(
        ctx: *mut StrataCtx,
        head: *mut f32,
        len: i64,
        pos: i64,
        n_rot: i64,
        head_dim: i64,
        freq_base: f64,
    ) -> c_int;
    pub(crate) fn strata_cuda_add(ctx: *mut StrataCtx, a: *mut f32, b: *const f32, n: i64) -> c_int;
    pub(crate) fn strata_cuda_rms_norm_dev(
        ctx: *mut StrataCtx,
        x_dev: *mut f32,
        w_dev: *const f32,
        n: i64,
        rows: i64,
        eps: f64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_l2_norm_dev(
        ctx: *mut StrataCtx,
        x_dev: *mut f32,
        head_dim: i64,
        heads: i64,
        eps: f64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_softmax_dev(
        ctx: *mut StrataCtx,
        x_dev: *mut f32,
        n: i64,
        rows: i64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_rope_neox_dev(
        ctx: *mut StrataCtx,
        x_dev: *mut f32,
        head_dim: i64,
        heads: i64,
        n_rot: i64,
        pos: i64,
        freq_base: f64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_add_dev(
        ctx: *mut StrataCtx,
        a_dev: *mut f32,
        b_dev: *const f32,
        n: i64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_comm_unique_id(id_out: *mut u8) -> c_int;
    pub(crate) fn strata_cuda_comm_init(ctx: *mut StrataCtx, rank: c_int, world: c_int, id: *const u8) -> c_int;
    pub(crate) fn strata_cuda_comm_info(ctx: *const StrataCtx, rank: *mut c_int, world: *mut c_int) -> c_int;
    pub(crate) fn strata_cuda_comm_group_start(ctx: *mut StrataCtx) -> c_int;
    pub(crate) fn strata_cuda_comm_group_end(ctx: *mut StrataCtx) -> c_int;
    pub(crate) fn strata_cuda_gemv_sharded_dev(
        ctx: *mut StrataCtx,
        w_shard: *const StrataWeight,
        x_dev: *const f32,
        y_dev: *mut f32,
        batch: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemm_sharded_dev(
        ctx: *mut StrataCtx,
        w_shard: *const StrataWeight,
        x_dev: *const u16,
        y_dev: *mut f32,
        m: i64,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_comm_set_gather(ctx: *mut StrataCtx, mode: c_int) -> c_int;
    pub(crate) fn strata_cuda_comm_peer_info(
        ctx: *const StrataCtx,
        available: *mut c_int,
        capacity_floats: *mut i64,
    ) -> c_int;
    pub(crate) fn strata_cuda_moe_ffn_ep_dev(
        ctx: *mut StrataCtx,
        layer: *const StrataMoe,
        x_dev: *const f32,
        router_logits_dev: *const f32,
        tokens: i64,
        out_dev: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemv_noalloc(
        w_dev: *const u8,
        quant: u32,
        rows: i64,
        cols: i64,
        x_dev: *const f32,
        y_dev: *mut f32,
        batch: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub(crate) fn strata_cuda_gemv_noalloc_status(stream: *mut c_void, clear: c_int) -> c_int;
}

// include/strata_gguf.h
extern "C" {
    pub(crate) fn strata_cuda_gguf_open(
        any_shard: *const c_char,
        out: *mut *mut StrataGguf,
        err: *mut c_char,
        err_len: usize,
    ) -> c_int;
    pub(crate) fn strata_cuda_gguf_close(g: *mut StrataGguf);
    pub(crate) fn strata_cuda_gguf_split_paths(
        any_shard: *const c_char,
        buf: *mut c_char,
        buf_len: usize,
        needed: *mut usize,
        err: *mut c_char,
        err_len: usize,
    ) -> c_int;
    pub(crate) fn strata_cuda_gguf_n_shards(g: *const StrataGguf) -> c_int;
    pub(crate) fn strata_cuda_gguf_shard(g: *const StrataGguf, shard: c_int, out: *mut strata_gguf_shard) -> c_int;
    pub(crate) fn strata_cuda_gguf_tensor_count(g: *const StrataGguf) -> i64;
    pub(crate) fn strata_cuda_gguf_tensor(g: *const StrataGguf, index: i64, out: *mut strata_gguf_tensor) -> c_int;
    pub(crate) fn strata_cuda_gguf_find(g: *const StrataGguf, name: *const c_char, index: *mut i64) -> c_int;
    pub(crate) fn strata_cuda_gguf_tensor_data(
        g: *const StrataGguf,
        index: i64,
        data: *mut *const u8,
        nbytes: *mut u64,
        err: *mut c_char,
        err_len: usize,
    ) -> c_int;
    pub(crate) fn strata_cuda_gguf_meta(g: *const StrataGguf, key: *const c_char, out: *mut strata_gguf_value) -> c_int;
    pub(crate) fn strata_cuda_gguf_view(
        g: *const StrataGguf,
        index: i64,
        first: i64,
        count: i64,
        out: *mut strata_upload,
        err: *mut c_char,
        err_len: usize,
    ) -> c_int;
    pub(crate) fn strata_cuda_gguf_ingest(
        ctx: *mut StrataCtx,
        g: *const StrataGguf,
        tensors: *const i64,
        n: i64,
        out: *mut *mut StrataWeight,
    ) -> c_int;
    pub(crate) fn strata_cuda_gguf_moe_layer(
        ctx: *mut StrataCtx,
        g: *const StrataGguf,
        layer: i64,
        top_k: i64,
        expert_begin: i64,
        expert_end: i64,
        with_shared: c_int,
        out: *mut *mut StrataMoe,
        weights_out: *mut *mut StrataWeight,
    ) -> c_int;
}
