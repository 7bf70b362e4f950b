"""Python binding of libstrata_cuda.so (the C ABI in include/strata_cuda.h).

This is the host-side mirror of strata-core's ComputeBackend seam
(crates/strata-core/src/backend.rs:20-51) for Python callers, tests and the
benchmark: `CudaBackend.gemv` / `expert_gemv` take the same arguments and
meaning as the trait methods (a QuantTensor or ExpertView, host f32 slices,
an unused scratch), and failures raise `BackendError` carrying the status
code, as `strata_core::Error::Backend` would.

There is no fallback: if the shared library is missing or no CUDA device is
present, construction raises.
"""
from __future__ import annotations

import ctypes as C
import os
from collections import OrderedDict
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("STRATA_CUDA_LIB", HERE / "libstrata_cuda.so"))

# status codes (include/strata_cuda.h)
(OK, ERR_INVALID, ERR_UNSUPPORTED_QUANT, ERR_TRUNCATED, ERR_CUDA, ERR_OOM, ERR_TIMEOUT, ERR_NCCL, ERR_BUDGET,
 ERR_SCRATCH_LIMIT) = range(10)
# include/strata_gguf.h: one per strata_gguf::Error variant the reader raises
(ERR_IO, ERR_BAD_MAGIC, ERR_UNSUPPORTED_VERSION, ERR_BAD_VALUE_TYPE, ERR_BAD_KEY_LENGTH, ERR_STRING_NOT_UTF8,
 ERR_TENSOR_NOT_FOUND, ERR_WRONG_TENSOR_DIMS) = range(10, 18)

# Strata ggml type ids (crates/strata-gguf/src/quant.rs:15-43)
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 8, 12, 13, 14, 30
Q4_0, Q4_1, Q5_0, Q5_1, Q8_1, Q2_K, Q3_K, IQ4_NL, IQ4_XS, MXFP4, NVFP4, Q2_0 = 2, 3, 6, 7, 9, 10, 11, 20, 23, 39, 40, 42
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176),
         Q6_K: (256, 210), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), Q8_1: (32, 36),
         Q2_K: (256, 84), Q3_K: (256, 110), IQ4_NL: (32, 18), IQ4_XS: (256, 136), MXFP4: (32, 17),
         NVFP4: (64, 36), Q2_0: (64, 18)}
NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K",
         Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1", Q8_1: "Q8_1", Q2_K: "Q2_K", Q3_K: "Q3_K",
         IQ4_NL: "IQ4_NL", IQ4_XS: "IQ4_XS", MXFP4: "MXFP4", NVFP4: "NVFP4", Q2_0: "Q2_0"}


def byte_size(quant: int, n: int) -> int:
    """QuantType::byte_size (crates/strata-gguf/src/quant.rs:178-180)."""
    bs, ts = BLOCK[quant]
    return -(-n // bs) * ts


class BackendError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Loads libstrata_cuda.so once; raises if it is not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is not built (run strata-rs_b200/build.py)")
        L = C.CDLL(str(LIB_PATH))
        vp, i32, i64, u32, u64, sz = C.c_void_p, C.c_int, C.c_int64, C.c_uint32, C.c_uint64, C.c_size_t
        fp = C.POINTER(C.c_float)
        sig = {
            "strata_cuda_abi_version": (i32, []),
            "strata_cuda_name": (C.c_char_p, []),
            "strata_cuda_create": (i32, [i32, C.POINTER(vp)]),
            "strata_cuda_destroy": (i32, [vp]),
            "strata_cuda_last_error": (C.c_char_p, [vp]),
            "strata_cuda_set_weight_budget": (i32, [vp, u64]),
            "strata_cuda_resident_bytes": (i32, [vp, C.POINTER(u64)]),
            "strata_cuda_set_wait_timeout_ms": (i32, [vp, u32]),
            "strata_cuda_synchronize": (i32, [vp]),
            "strata_cuda_set_gemv_path": (i32, [vp, i32]),
            "strata_cuda_stream": (i32, [vp, C.POINTER(vp)]),
            "strata_cuda_upload": (i32, [vp, vp, sz, u32, i64, i64, i64, C.POINTER(vp)]),
            "strata_cuda_upload_many": (i32, [vp, C.POINTER(UploadItem), i64, C.POINTER(vp)]),
            "strata_cuda_gguf_open": (i32, [C.c_char_p, C.POINTER(vp), C.c_char_p, sz]),
            "strata_cuda_gguf_close": (None, [vp]),
            "strata_cuda_gguf_split_paths": (i32, [C.c_char_p, C.c_char_p, sz, C.POINTER(sz), C.c_char_p, sz]),
            "strata_cuda_gguf_n_shards": (i32, [vp]),
            "strata_cuda_gguf_shard": (i32, [vp, i32, C.POINTER(GgufShardInfo)]),
            "strata_cuda_gguf_tensor_count": (i64, [vp]),
            "strata_cuda_gguf_tensor": (i32, [vp, i64, C.POINTER(GgufTensorInfo)]),
            "strata_cuda_gguf_find": (i32, [vp, C.c_char_p, C.POINTER(i64)]),
            "strata_cuda_gguf_tensor_data": (i32, [vp, i64, C.POINTER(vp), C.POINTER(u64), C.c_char_p, sz]),
            "strata_cuda_gguf_meta": (i32, [vp, C.c_char_p, C.POINTER(GgufValue)]),
            "strata_cuda_gguf_ingest": (i32, [vp, vp, C.POINTER(i64), i64, C.POINTER(vp)]),
            "strata_cuda_gguf_view": (i32, [vp, i64, i64, i64, C.POINTER(UploadItem), C.c_char_p, sz]),
            "strata_cuda_gguf_moe_layer": (i32, [vp, vp, i64, i64, i64, i64, i32, C.POINTER(vp), C.POINTER(vp)]),
            "strata_cuda_free_weight": (i32, [vp]),
            "strata_cuda_dequant": (i32, [vp, vp, i64, i64, i64, fp]),
            "strata_cuda_gemv": (i32, [vp, vp, fp, fp, i32]),
            "strata_cuda_gemv_dev": (i32, [vp, vp, vp, vp, i32, vp]),
            "strata_cuda_expert_gemv": (i32, [vp, vp, i64, fp, fp, i32]),
            "strata_cuda_expert_gemv_dev": (i32, [vp, vp, i64, vp, vp, i32, vp]),
            "strata_cuda_gemv_noalloc": (i32, [vp, u32, i64, i64, vp, vp, i32, vp]),
            "strata_cuda_gemv_noalloc_status": (i32, [vp, i32]),
            "strata_cuda_gemm_bf16": (i32, [vp, vp, vp, fp, i64]),
            "strata_cuda_gemm_bf16_dev": (i32, [vp, vp, vp, vp, i64, vp]),
            "strata_cuda_gemm_f32": (i32, [vp, vp, fp, fp, i64]),
            "strata_cuda_gemm_f32_dev": (i32, [vp, vp, vp, vp, i64, vp]),
            "strata_cuda_set_gemm_terms": (i32, [vp, i32]),
            "strata_cuda_moe_create": (i32, [vp, C.POINTER(MoeDesc), C.POINTER(vp)]),
            "strata_cuda_moe_destroy": (i32, [vp]),
            "strata_cuda_moe_ffn": (i32, [vp, vp, fp, fp, i64, fp, C.POINTER(C.c_int32), fp]),
            "strata_cuda_moe_ffn_dev": (i32, [vp, vp, vp, vp, i64, vp, vp, vp, vp]),
            "strata_cuda_comm_unique_id": (i32, [vp]),
            "strata_cuda_comm_init": (i32, [vp, i32, i32, vp]),
            "strata_cuda_comm_info": (i32, [vp, C.POINTER(i32), C.POINTER(i32)]),
            "strata_cuda_comm_group_start": (i32, [vp]),
            "strata_cuda_comm_group_end": (i32, [vp]),
            "strata_cuda_comm_set_gather": (i32, [vp, i32]),
            "strata_cuda_rms_norm": (i32, [vp, fp, fp, i64, C.c_double]),
            "strata_cuda_l2_norm": (i32, [vp, fp, i64, C.c_double]),
            "strata_cuda_softmax": (i32, [vp, fp, i64]),
            "strata_cuda_rope_neox": (i32, [vp, fp, i64, i64, i64, i64, C.c_double]),
            "strata_cuda_add": (i32, [vp, fp, fp, i64]),
            "strata_cuda_rms_norm_dev": (i32, [vp, vp, vp, i64, i64, C.c_double, vp]),
            "strata_cuda_l2_norm_dev": (i32, [vp, vp, i64, i64, C.c_double, vp]),
            "strata_cuda_softmax_dev": (i32, [vp, vp, i64, i64, vp]),
            "strata_cuda_rope_neox_dev": (i32, [vp, vp, i64, i64, i64, i64, C.c_double, vp]),
            "strata_cuda_add_dev": (i32, [vp, vp, vp, i64, vp]),
            "strata_cuda_comm_peer_info": (i32, [vp, C.POINTER(i32), C.POINTER(i64)]),
            "strata_cuda_gemv_sharded_dev": (i32, [vp, vp, vp, vp, i32, vp]),
            "strata_cuda_gemm_sharded_dev": (i32, [vp, vp, vp, vp, i64, vp]),
            "strata_cuda_moe_ffn_ep_dev": (i32, [vp, vp, vp, vp, i64, vp, vp]),
        }
        for name, (res, args) in sig.items():
            if not hasattr(L, name):
                continue
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _lib = L
    return _lib


class MoeDesc(C.Structure):
    """strata_moe_desc (strata_cuda.h)."""
    _fields_ = [(nm, C.c_void_p) for nm in ("router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp",
                                            "down_shexp", "gate_inp_shexp")]
    _fields_ += [(nm, C.c_int64) for nm in ("n_embd", "n_expert", "top_k", "n_ff", "n_ff_shexp", "expert_begin",
                                            "expert_end")]
    _fields_ += [("with_shared", C.c_int)]


class UploadItem(C.Structure):
    """strata_upload (strata_cuda.h)."""
    _fields_ = [("bytes", C.c_void_p), ("len", C.c_size_t), ("quant", C.c_uint32), ("n_expert", C.c_int64),
                ("rows", C.c_int64), ("cols", C.c_int64)]


class GgufShardInfo(C.Structure):
    """strata_gguf_shard (strata_gguf.h)."""
    _fields_ = [("path", C.c_char_p), ("version", C.c_uint32), ("alignment", C.c_uint64),
                ("data_start", C.c_uint64), ("file_size", C.c_uint64), ("n_tensors", C.c_int64),
                ("n_metadata", C.c_int64)]


class GgufTensorInfo(C.Structure):
    """strata_gguf_tensor (strata_gguf.h)."""
    _fields_ = [("name", C.c_void_p), ("name_len", C.c_uint64), ("type", C.c_uint32), ("n_dims", C.c_int32),
                ("dims", C.c_uint64 * 4), ("offset", C.c_uint64), ("shard", C.c_int32)]


class GgufValue(C.Structure):
    """strata_gguf_value (strata_gguf.h)."""
    _fields_ = [("type", C.c_uint32), ("i", C.c_int64), ("u", C.c_uint64), ("f", C.c_double),
                ("str", C.c_void_p), ("str_len", C.c_uint64), ("elem", C.c_uint32), ("count", C.c_uint64)]


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


@dataclass
class QuantTensor:
    """strata_core::backend::QuantTensor (backend.rs:114-154): rows = OUT, cols = IN."""
    name: str
    quant: int
    rows: int
    cols: int
    data: np.ndarray  # uint8

    def row_bytes(self) -> int:
        return byte_size(self.quant, self.cols)


@dataclass
class ExpertView:
    """strata_core::weights::ExpertView (weights.rs:11-34): [n_expert][rows = IN][cols = OUT]."""
    name: str
    quant: int
    n_expert: int
    rows: int
    cols: int
    data: np.ndarray  # uint8


class Weight:
    """A tensor resident in HBM (uploaded byte-for-byte)."""

    def __init__(self, ctx: "Context", handle: C.c_void_p, quant: int, n_expert: int, rows: int, cols: int):
        self.ctx, self.handle, self.quant = ctx, handle, quant
        self.n_expert, self.rows, self.cols = n_expert, rows, cols

    def free(self):
        if self.handle and self.ctx.h:  # a closed context has released its weights already
            lib().strata_cuda_free_weight(self.handle)
        self.handle = None


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for strata_cuda_comm_init."""
    buf = C.create_string_buffer(128)
    rc = lib().strata_cuda_comm_unique_id(buf)
    if rc != OK:
        raise BackendError(rc, "strata_cuda_comm_unique_id failed")
    return buf.raw


@dataclass
class GgufTensor:
    """strata_gguf::TensorInfo (crates/strata-gguf/src/reader.rs:179-199) plus the shard holding it."""
    name: str
    shape: list
    ty: int
    offset: int
    shard: int


@dataclass
class MetaValue:
    """strata_gguf::MetaValue (crates/strata-gguf/src/metadata.rs:51-111) without array items."""
    ty: int
    int: int
    uint: int
    float: float
    string: str
    elem: int
    count: int

    def as_int(self):
        return self.int if self.ty not in (6, 8, 9, 12) else None

    def as_float(self):
        if self.ty in (8, 9):
            return None
        return self.float if self.ty in (6, 12) else float(self.int)

    def as_str(self):
        return self.string if self.ty == 8 else None


def split_paths(any_shard: str) -> list:
    """strata_gguf::split_paths (crates/strata-gguf/src/reader.rs:527-572)."""
    err = C.create_string_buffer(1024)
    need = C.c_size_t()
    L = lib()
    rc = L.strata_cuda_gguf_split_paths(str(any_shard).encode(), None, 0, C.byref(need), err, len(err))
    if rc not in (OK, ERR_INVALID) or (rc == ERR_INVALID and need.value == 0):
        raise BackendError(rc, err.value.decode())
    buf = C.create_string_buffer(need.value)
    rc = L.strata_cuda_gguf_split_paths(str(any_shard).encode(), buf, len(buf), C.byref(need), err, len(err))
    if rc != OK:
        raise BackendError(rc, err.value.decode())
    return buf.value.decode().splitlines()


class GgufModel:
    """strata_gguf::GgufModel (crates/strata-gguf/src/reader.rs:448-523): every shard of a
    model, mapped read-only, with one name index. Needs no GPU. Errors raise
    BackendError with the strata_gguf::Error code and text."""

    def __init__(self, any_shard):
        err = C.create_string_buffer(1024)
        h = C.c_void_p()
        rc = lib().strata_cuda_gguf_open(str(any_shard).encode(), C.byref(h), err, len(err))
        if rc != OK:
            raise BackendError(rc, err.value.decode())
        self.h = h

    def close(self):
        if self.h:
            lib().strata_cuda_gguf_close(self.h)
            self.h = None

    def __del__(self):  # unmaps the shards of a model nobody closed
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def n_shards(self) -> int:
        return lib().strata_cuda_gguf_n_shards(self.h)

    def shard(self, i: int) -> dict:
        info = GgufShardInfo()
        rc = lib().strata_cuda_gguf_shard(self.h, i, C.byref(info))
        if rc != OK:
            raise BackendError(rc, f"no shard {i}")
        return {k: (getattr(info, k).decode() if k == "path" else getattr(info, k)) for k, _ in info._fields_}

    def tensor_count(self) -> int:
        return lib().strata_cuda_gguf_tensor_count(self.h)

    def tensor(self, index: int) -> GgufTensor:
        t = GgufTensorInfo()
        rc = lib().strata_cuda_gguf_tensor(self.h, index, C.byref(t))
        if rc != OK:
            raise BackendError(rc, f"no tensor {index}")
        name = C.string_at(t.name, t.name_len).decode()
        return GgufTensor(name, list(t.dims[:t.n_dims]), t.type, t.offset, t.shard)

    def tensors(self) -> list:
        return [self.tensor(i) for i in range(self.tensor_count())]

    def index_of(self, name: str) -> int:
        """The tensor's position, or -1 when absent (GgufModel::find)."""
        i = C.c_int64()
        lib().strata_cuda_gguf_find(self.h, name.encode(), C.byref(i))
        return i.value

    def find(self, name: str):
        i = self.index_of(name)
        return None if i < 0 else self.tensor(i)

    def tensor_data(self, name_or_index) -> np.ndarray:
        """The payload bytes as a read-only view of the mapping (valid while the model is open)."""
        i = self.index_of(name_or_index) if isinstance(name_or_index, str) else name_or_index
        if i < 0:
            raise BackendError(ERR_TENSOR_NOT_FOUND, f"tensor '{name_or_index}' is missing from the file")
        p, n = C.c_void_p(), C.c_uint64()
        err = C.create_string_buffer(1024)
        rc = lib().strata_cuda_gguf_tensor_data(self.h, i, C.byref(p), C.byref(n), err, len(err))
        if rc != OK:
            raise BackendError(rc, err.value.decode())
        if n.value == 0:
            return np.zeros(0, np.uint8)
        a = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n.value,))
        a.flags.writeable = False
        return a

    def view(self, name_or_index, first: int = 0, count: int = -1) -> UploadItem:
        """strata_cuda_gguf_view: the upload item for rows (1-D / 2-D) or experts (3-D)
        [first, first + count) of a tensor, pointing into the mapping."""
        i = self.index_of(name_or_index) if isinstance(name_or_index, str) else name_or_index
        if i < 0:
            raise BackendError(ERR_TENSOR_NOT_FOUND, f"tensor '{name_or_index}' is missing from the file")
        u = UploadItem()
        err = C.create_string_buffer(1024)
        rc = lib().strata_cuda_gguf_view(self.h, i, first, count, C.byref(u), err, len(err))
        if rc != OK:
            raise BackendError(rc, err.value.decode())
        return u

    def get(self, key: str):
        """A metadata value of the first shard (GgufModel::get), or None."""
        v = GgufValue()
        if lib().strata_cuda_gguf_meta(self.h, key.encode(), C.byref(v)) != OK:
            return None
        s = C.string_at(v.str, v.str_len).decode() if v.str_len else ""
        return MetaValue(v.type, v.i, v.u, v.f, s, v.elem, v.count)


class MoeLayer:
    def __init__(self, ctx: "Context", handle: C.c_void_p, n_embd: int, n_expert: int, top_k: int):
        self.ctx, self.handle = ctx, handle
        self.n_embd, self.n_expert, self.top_k = n_embd, n_expert, top_k

    def free(self):
        if self.handle:
            lib().strata_cuda_moe_destroy(self.handle)
            self.handle = None


class Context:
    """One device + stream (strata_cuda_create)."""

    def __init__(self, device: int = 0):
        L = lib()
        h = C.c_void_p()
        rc = L.strata_cuda_create(device, C.byref(h))
        if rc != OK:
            raise BackendError(rc, f"strata_cuda_create(device={device}) failed")
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().strata_cuda_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def check(self, rc: int):
        if rc != OK:
            raise BackendError(rc, lib().strata_cuda_last_error(self.h).decode())

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        self.check(lib().strata_cuda_stream(self.h, C.byref(s)))
        return s.value or 0

    GEMV_AUTO, GEMV_CUDA_CORES, GEMV_TENSOR_CORES = 0, 1, 2

    def set_gemv_path(self, path: int):
        self.check(lib().strata_cuda_set_gemv_path(self.h, path))

    def synchronize(self):
        self.check(lib().strata_cuda_synchronize(self.h))

    def set_weight_budget(self, nbytes: int):
        self.check(lib().strata_cuda_set_weight_budget(self.h, nbytes))

    def set_wait_timeout_ms(self, ms: int):
        self.check(lib().strata_cuda_set_wait_timeout_ms(self.h, ms))

    def resident_bytes(self) -> int:
        v = C.c_uint64()
        self.check(lib().strata_cuda_resident_bytes(self.h, C.byref(v)))
        return v.value

    def upload(self, data: np.ndarray, quant: int, rows: int, cols: int, n_expert: int = 0) -> Weight:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        h = C.c_void_p()
        self.check(lib().strata_cuda_upload(self.h, data.ctypes.data, data.nbytes, quant, n_expert, rows, cols,
                                            C.byref(h)))
        return Weight(self, h, quant, n_expert, rows, cols)

    def upload_many(self, items: list) -> list:
        """strata_cuda_upload_many: items are (data, quant, rows, cols, n_expert) tuples."""
        arrs = [np.ascontiguousarray(d, dtype=np.uint8) for d, *_ in items]
        descs = (UploadItem * max(1, len(items)))()
        for k, (a, (_, quant, rows, cols, n_expert)) in enumerate(zip(arrs, items)):
            descs[k] = UploadItem(a.ctypes.data, a.nbytes, quant, n_expert, rows, cols)
        hs = (C.c_void_p * max(1, len(items)))()
        self.check(lib().strata_cuda_upload_many(self.h, descs, len(items), hs))
        return [Weight(self, C.c_void_p(hs[k]), q, ne, r, c) for k, (_, q, r, c, ne) in enumerate(items)]

    def upload_views(self, views: list) -> list:
        """strata_cuda_upload_many over UploadItems (GgufModel.view): the bytes stay in the mapping."""
        items = (UploadItem * max(1, len(views)))(*views)
        hs = (C.c_void_p * max(1, len(views)))()
        self.check(lib().strata_cuda_upload_many(self.h, items, len(views), hs))
        return [Weight(self, C.c_void_p(hs[k]), v.quant, v.n_expert, v.rows, v.cols) for k, v in enumerate(views)]

    def ingest(self, model: GgufModel, names: list) -> dict:
        """strata_cuda_gguf_ingest: the named tensors of an opened model, as WeightStore views them."""
        idx = []
        for nm in names:
            i = model.index_of(nm)
            if i < 0:
                raise BackendError(ERR_TENSOR_NOT_FOUND, f"tensor '{nm}' is missing from the file")
            idx.append(i)
        ix = (C.c_int64 * max(1, len(idx)))(*idx)
        hs = (C.c_void_p * max(1, len(idx)))()
        self.check(lib().strata_cuda_gguf_ingest(self.h, model.h, ix, len(idx), hs))
        out = {}
        for k, nm in enumerate(names):
            t = model.tensor(idx[k])
            d = t.shape + [1] * (3 - len(t.shape))
            n_expert = d[2] if len(t.shape) == 3 else 0
            rows = 1 if len(t.shape) == 1 else d[1]
            out[nm] = Weight(self, C.c_void_p(hs[k]), t.ty, n_expert, rows, d[0])
        return out

    def dequant(self, w: Weight, row0: int = 0, nrows: int | None = None, expert: int = 0) -> np.ndarray:
        nrows = w.rows - row0 if nrows is None else nrows
        out = np.empty((nrows, w.cols), np.float32)
        self.check(lib().strata_cuda_dequant(self.h, w.handle, expert, row0, nrows, _fptr(out)))
        return out

    def gemv(self, w: Weight, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        batch = 1 if x.ndim == 1 else x.shape[0]
        y = np.empty((batch, w.rows), np.float32)
        self.check(lib().strata_cuda_gemv(self.h, w.handle, _fptr(x), _fptr(y), batch))
        return y[0] if x.ndim == 1 else y

    def expert_gemv(self, w: Weight, e: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        batch = 1 if x.ndim == 1 else x.shape[0]
        y = np.empty((batch, w.cols), np.float32)
        self.check(lib().strata_cuda_expert_gemv(self.h, w.handle, e, _fptr(x), _fptr(y), batch))
        return y[0] if x.ndim == 1 else y

    def gemm_bf16(self, w: Weight, x_bits: np.ndarray) -> np.ndarray:
        """Prefill GEMM: x_bits is m x cols bf16 bit patterns (uint16); returns m x rows f32."""
        x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
        m = x_bits.shape[0]
        y = np.empty((m, w.rows), np.float32)
        self.check(lib().strata_cuda_gemm_bf16(self.h, w.handle, x_bits.ctypes.data, _fptr(y), m))
        return y

    def gemm_f32(self, w: Weight, x: np.ndarray) -> np.ndarray:
        """Prefill GEMM on f32 activations (rounded to bf16 on the device)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        m = x.shape[0]
        y = np.empty((m, w.rows), np.float32)
        self.check(lib().strata_cuda_gemm_f32(self.h, w.handle, _fptr(x), _fptr(y), m))
        return y

    def moe_create(self, weights: dict, n_embd: int, n_expert: int, top_k: int, n_ff: int, n_ff_shexp: int = 0,
                   expert_begin: int = 0, expert_end: int | None = None, with_shared: bool = True) -> "MoeLayer":
        """weights maps MoeLayer field names (router, gate_exps, ...) to uploaded Weights."""
        d = MoeDesc()
        for nm in ("router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp", "down_shexp",
                   "gate_inp_shexp"):
            w = weights.get(nm)
            h = w.handle if w is not None else None
            setattr(d, nm, h.value if isinstance(h, C.c_void_p) else h)
        d.n_embd, d.n_expert, d.top_k, d.n_ff, d.n_ff_shexp = n_embd, n_expert, top_k, n_ff, n_ff_shexp
        d.expert_begin = expert_begin
        d.expert_end = n_expert if expert_end is None else expert_end
        d.with_shared = 1 if with_shared else 0
        h = C.c_void_p()
        self.check(lib().strata_cuda_moe_create(self.h, C.byref(d), C.byref(h)))
        return MoeLayer(self, h, n_embd, n_expert, top_k)

    def gguf_moe_layer(self, model: "GgufModel", layer: int, top_k: int, expert_begin: int = 0,
                       expert_end: int = 0, with_shared: bool = True):
        """strata_cuda_gguf_moe_layer (load_layer, crates/strata-core/src/moe.rs:147-188):
        returns the MoeLayer and its uploaded weights (free them after the layer)."""
        h = C.c_void_p()
        ws = (C.c_void_p * 8)()
        self.check(lib().strata_cuda_gguf_moe_layer(self.h, model.h, layer, top_k, expert_begin, expert_end,
                                                    1 if with_shared else 0, C.byref(h), ws))
        router = model.find(f"blk.{layer}.ffn_gate_inp.weight")
        exps = model.find(f"blk.{layer}.ffn_gate_exps.weight")
        weights = [Weight(self, C.c_void_p(p), 0, 0, 0, 0) for p in ws if p]
        return MoeLayer(self, h, router.shape[0], exps.shape[2], top_k), weights

    def moe_ffn(self, layer: "MoeLayer", x: np.ndarray, logits: np.ndarray | None = None):
        """MoE layer for each row of x (tokens x n_embd) -> (out, ids, weights)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, layer.n_embd)
        T = x.shape[0]
        lg = None
        if logits is not None:
            lg = np.ascontiguousarray(logits, dtype=np.float32).reshape(T, layer.n_expert)
        out = np.empty((T, layer.n_embd), np.float32)
        ids = np.empty((T, layer.top_k), np.int32)
        w = np.empty((T, layer.top_k), np.float32)
        self.check(lib().strata_cuda_moe_ffn(self.h, layer.handle, _fptr(x), _fptr(lg) if lg is not None else None, T,
                                             _fptr(out), ids.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(w)))
        return out, ids, w

    def moe_ffn_dev(self, layer: "MoeLayer", x_ptr: int, logits_ptr: int, tokens: int, out_ptr: int,
                    ids_ptr: int = 0, wts_ptr: int = 0, stream: int = 0):
        self.check(lib().strata_cuda_moe_ffn_dev(self.h, layer.handle, x_ptr, logits_ptr or None, tokens, out_ptr,
                                                 ids_ptr or None, wts_ptr or None, stream or None))

    # multi-GPU (one context per process and GPU)
    def comm_init(self, rank: int, world: int, uid: bytes):
        buf = C.create_string_buffer(bytes(uid), 128)
        self.check(lib().strata_cuda_comm_init(self.h, rank, world, buf))

    def comm_info(self) -> tuple[int, int]:
        r, w = C.c_int(), C.c_int()
        self.check(lib().strata_cuda_comm_info(self.h, C.byref(r), C.byref(w)))
        return r.value, w.value

    def comm_group_start(self):
        self.check(lib().strata_cuda_comm_group_start(self.h))

    def comm_group_end(self):
        self.check(lib().strata_cuda_comm_group_end(self.h))

    # ---- the elementwise trait methods (host slices, one vector per call)

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True).reshape(-1)
        w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
        if w.size < x.size:  # ops::rms_norm indexes w[i] for every i of x (a panic there)
            raise BackendError(ERR_INVALID, f"rms_norm: {w.size} weights for {x.size} values")
        self.check(lib().strata_cuda_rms_norm(self.h, _fptr(x), _fptr(w), x.size, eps))
        return x

    def l2_norm(self, head: np.ndarray, eps: float) -> np.ndarray:
        x = np.array(head, dtype=np.float32, copy=True).reshape(-1)
        self.check(lib().strata_cuda_l2_norm(self.h, _fptr(x), x.size, eps))
        return x

    def softmax(self, xs: np.ndarray) -> np.ndarray:
        x = np.array(xs, dtype=np.float32, copy=True).reshape(-1)
        self.check(lib().strata_cuda_softmax(self.h, _fptr(x), x.size))
        return x

    def rope_neox(self, head: np.ndarray, pos: int, n_rot: int, head_dim: int, freq_base: float) -> np.ndarray:
        x = np.array(head, dtype=np.float32, copy=True).reshape(-1)
        self.check(lib().strata_cuda_rope_neox(self.h, _fptr(x), x.size, pos, n_rot, head_dim, freq_base))
        return x

    def add(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        """a + b over the common length, a's tail unchanged (ops::add_into zips the two)."""
        x = np.array(a, dtype=np.float32, copy=True).reshape(-1)
        bb = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
        n = min(x.size, bb.size)
        if n:
            self.check(lib().strata_cuda_add(self.h, _fptr(x), _fptr(bb), n))
        return x

    # ---- the same on device pointers, many vectors per call

    def rms_norm_dev(self, x_ptr: int, w_ptr: int, n: int, rows: int, eps: float, stream: int = 0):
        self.check(lib().strata_cuda_rms_norm_dev(self.h, x_ptr, w_ptr, n, rows, eps, stream or None))

    def l2_norm_dev(self, x_ptr: int, head_dim: int, heads: int, eps: float, stream: int = 0):
        self.check(lib().strata_cuda_l2_norm_dev(self.h, x_ptr, head_dim, heads, eps, stream or None))

    def softmax_dev(self, x_ptr: int, n: int, rows: int, stream: int = 0):
        self.check(lib().strata_cuda_softmax_dev(self.h, x_ptr, n, rows, stream or None))

    def rope_neox_dev(self, x_ptr: int, head_dim: int, heads: int, n_rot: int, pos: int, freq_base: float,
                      stream: int = 0):
        self.check(lib().strata_cuda_rope_neox_dev(self.h, x_ptr, head_dim, heads, n_rot, pos, freq_base,
                                                   stream or None))

    def add_dev(self, a_ptr: int, b_ptr: int, n: int, stream: int = 0):
        self.check(lib().strata_cuda_add_dev(self.h, a_ptr, b_ptr, n, stream or None))

    GATHER_AUTO, GATHER_NCCL, GATHER_PEER = 0, 1, 2

    def comm_set_gather(self, mode: int):
        """How sharded GEMVs gather rows: GATHER_AUTO, GATHER_NCCL or GATHER_PEER
        (the all-gather fused into the GEMV's epilogue over peer memory)."""
        self.check(lib().strata_cuda_comm_set_gather(self.h, mode))

    def comm_peer_info(self) -> tuple[bool, int]:
        """(peer gather available on every rank, its capacity in floats)."""
        a, cap = C.c_int32(), C.c_int64()
        self.check(lib().strata_cuda_comm_peer_info(self.h, C.byref(a), C.byref(cap)))
        return bool(a.value), cap.value

    def gemv_sharded_dev(self, w: Weight, x_ptr: int, y_ptr: int, batch: int, stream: int = 0):
        self.check(lib().strata_cuda_gemv_sharded_dev(self.h, w.handle, x_ptr, y_ptr, batch, stream or None))

    def gemm_sharded_dev(self, w: Weight, x_ptr: int, y_ptr: int, m: int, stream: int = 0):
        self.check(lib().strata_cuda_gemm_sharded_dev(self.h, w.handle, x_ptr, y_ptr, m, stream or None))

    def moe_ffn_ep_dev(self, layer: "MoeLayer", x_ptr: int, logits_ptr: int, tokens: int, out_ptr: int,
                       stream: int = 0):
        self.check(lib().strata_cuda_moe_ffn_ep_dev(self.h, layer.handle, x_ptr, logits_ptr or None, tokens, out_ptr,
                                                    stream or None))

    def set_gemm_terms(self, terms: int):
        self.check(lib().strata_cuda_set_gemm_terms(self.h, terms))

    # device-pointer variants (int addresses, e.g. torch.Tensor.data_ptr())
    def gemm_bf16_dev(self, w: Weight, x_ptr: int, y_ptr: int, m: int, stream: int = 0):
        self.check(lib().strata_cuda_gemm_bf16_dev(self.h, w.handle, x_ptr, y_ptr, m, stream or None))

    def gemm_f32_dev(self, w: Weight, x_ptr: int, y_ptr: int, m: int, stream: int = 0):
        self.check(lib().strata_cuda_gemm_f32_dev(self.h, w.handle, x_ptr, y_ptr, m, stream or None))

    def gemv_dev(self, w: Weight, x_ptr: int, y_ptr: int, batch: int, stream: int = 0):
        self.check(lib().strata_cuda_gemv_dev(self.h, w.handle, x_ptr, y_ptr, batch, stream or None))

    def expert_gemv_dev(self, w: Weight, e: int, x_ptr: int, y_ptr: int, batch: int, stream: int = 0):
        self.check(lib().strata_cuda_expert_gemv_dev(self.h, w.handle, e, x_ptr, y_ptr, batch, stream or None))


@dataclass
class RopeCfg:
    """strata_core::backend::RopeCfg (crates/strata-core/src/backend.rs:158-167)."""
    pos: int
    n_rot: int
    head_dim: int
    freq_base: float


DEFAULT_WEIGHT_BUDGET = 4 << 30  # WgpuBackend::probe's default (crates/strata-backend-wgpu/src/gpu.rs:227-229)


class CudaBackend:
    """strata-core's ComputeBackend over the CUDA path (name() == "cuda").

    Weights are uploaded on first use and cached by (data address, length,
    n_expert), like the wgpu backend's cache (crates/strata-backend-wgpu/src/gpu.rs:271,287);
    as its WeightCache (gpu.rs:61-112), the cache holds at most `budget_bytes`
    of resident weights and evicts the least recently used first when a new
    weight would not fit (an entry larger than the budget is still uploaded).
    The CLI's --gpu-weights-mib (crates/strata-cli/src/main.rs:116-118) maps here.
    """

    def __init__(self, device: int = 0, budget_bytes: int = DEFAULT_WEIGHT_BUDGET):
        self.ctx = Context(device)
        self.budget = budget_bytes
        self._cache: OrderedDict[tuple[int, int, int], Weight] = OrderedDict()
        self._bytes = 0

    def name(self) -> str:
        return lib().strata_cuda_name().decode()

    def resident_bytes(self) -> int:
        """Bytes of weights the cache holds (WgpuBackend::resident_bytes)."""
        return self._bytes

    def _resident(self, data: np.ndarray, quant: int, rows: int, cols: int, n_expert: int) -> Weight:
        key = (data.ctypes.data, data.nbytes, n_expert)
        w = self._cache.get(key)
        if w is not None:
            self._cache.move_to_end(key)  # most recently used
            return w
        need = byte_size(quant, cols) * rows * max(1, n_expert) if quant in BLOCK else data.nbytes
        while self._cache and self._bytes + need > self.budget:
            _, victim = self._cache.popitem(last=False)
            self._bytes -= victim.cached_bytes
            victim.free()
        w = self.ctx.upload(data, quant, rows, cols, n_expert)
        w.cached_bytes = need
        self._cache[key] = w
        self._bytes += need
        return w

    def gemv(self, w: QuantTensor, x: np.ndarray, y: np.ndarray, scratch=None) -> None:
        if x.shape[-1] != w.cols or y.shape[-1] != w.rows:
            raise BackendError(ERR_INVALID, f"gemv {w.name}: x/y do not match {w.rows}x{w.cols}")
        dw = self._resident(w.data, w.quant, w.rows, w.cols, 0)
        y[...] = self.ctx.gemv(dw, x)

    def expert_gemv(self, w: ExpertView, e: int, x: np.ndarray, y: np.ndarray, scratch=None) -> None:
        if x.shape[-1] != w.rows or y.shape[-1] != w.cols:
            raise BackendError(ERR_INVALID, f"expert_gemv {w.name}: x/y do not match {w.rows}x{w.cols}")
        dw = self._resident(w.data, w.quant, w.rows, w.cols, w.n_expert)
        y[...] = self.ctx.expert_gemv(dw, e, x)

    # the elementwise trait methods (backend.rs:37-50), in place on the caller's slices
    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> None:
        x[...] = self.ctx.rms_norm(x, w, eps).reshape(x.shape)

    def rope_neox(self, head: np.ndarray, cfg: RopeCfg) -> None:
        head[...] = self.ctx.rope_neox(head, cfg.pos, cfg.n_rot, cfg.head_dim, cfg.freq_base).reshape(head.shape)

    def softmax(self, xs: np.ndarray) -> None:
        xs[...] = self.ctx.softmax(xs).reshape(xs.shape)

    def l2_norm(self, head: np.ndarray, eps: float) -> None:
        head[...] = self.ctx.l2_norm(head, eps).reshape(head.shape)

    def add(self, a: np.ndarray, b: np.ndarray) -> None:
        a[...] = self.ctx.add(a, b).reshape(a.shape)

    def close(self):
        for w in self._cache.values():
            w.free()
        self._cache.clear()
        self._bytes = 0
        self.ctx.close()
