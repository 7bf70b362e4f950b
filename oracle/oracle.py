"""ctypes binding of liboracle.so — the CPU restatement of strata-rs's path.

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it;
the product (libstrata_cuda.so and strata-rs_b200/*.py) never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SO = HERE / "liboracle.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_TRUNCATED = 0, 1, 2, 3


def build() -> Path:
    """Builds liboracle.so with oracle/Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return SO


_L = None


def lib() -> C.CDLL:
    global _L
    if _L is None:
        if not SO.exists():
            build()
        L = C.CDLL(str(SO))
        i64, u32, sz, i32 = C.c_int64, C.c_uint32, C.c_size_t, C.c_int
        fp, vp, lp = C.POINTER(C.c_float), C.c_void_p, C.POINTER(C.c_int64)
        sigs = {
            "orc_block_size": (i64, [u32]),
            "orc_type_size": (i64, [u32]),
            "orc_byte_size": (i64, [u32, i64]),
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_bf16_round": (C.c_float, [C.c_float]),
            "orc_f32_to_bf16_bits": (C.c_uint16, [C.c_float]),
            "orc_dequantize_row": (i32, [u32, vp, sz, fp, i64]),
            "orc_gemv": (i32, [u32, vp, sz, i64, i64, fp, fp]),
            "orc_gemv_batch": (i32, [u32, vp, sz, i64, i64, fp, fp, i64, i32]),
            "orc_gemv_rows": (i32, [u32, vp, sz, i64, i64, fp, fp, i64, i64, i32]),
            "orc_expert_gemv": (i32, [u32, vp, sz, i64, i64, i64, i64, fp, fp]),
            "orc_silu": (C.c_float, [C.c_float]),
            "orc_sigmoid": (C.c_float, [C.c_float]),
            "orc_moe_route_logits": (i32, [fp, i64, i64, lp, fp]),
            "orc_moe_route": (i32, [vp, fp, lp, fp]),
            "orc_moe_combine": (i32, [vp, fp, lp, fp, fp]),
            "orc_moe_layer": (i32, [vp, fp, fp, i64, fp, lp, fp, i32]),
            "orc_rms_norm": (None, [fp, fp, i64, C.c_double]),
            "orc_l2_norm": (None, [fp, i64, C.c_double]),
            "orc_softmax": (None, [fp, i64]),
            "orc_rope_neox": (None, [fp, i64, i64, i64, i64, C.c_double]),
            "orc_add": (None, [fp, fp, i64]),
            "orc_expf_misrounded": (i64, [C.c_float, C.c_float, fp, i64]),
            "orc_expf_tie_pairs": (i64, [C.c_float, C.c_float, fp, i64]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _L = L
    return _L


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _check(rc: int, what: str):
    if rc != OK:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


def dequantize_row(quant: int, block: np.ndarray, n: int) -> np.ndarray:
    block = np.ascontiguousarray(block, dtype=np.uint8)
    out = np.empty(n, np.float32)
    _check(lib().orc_dequantize_row(quant, block.ctypes.data, block.nbytes, _fp(out), n), "dequantize_row")
    return out


def dequantize(quant: int, data: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """All rows of a [rows][cols] tensor (row by row, like WeightStore::f32_vec)."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    rb = int(lib().orc_byte_size(quant, cols))
    out = np.empty((rows, cols), np.float32)
    for r in range(rows):
        out[r] = dequantize_row(quant, data[r * rb:(r + 1) * rb], cols)
    return out


def gemv(quant: int, data: np.ndarray, rows: int, cols: int, x: np.ndarray, threads: int = 1) -> np.ndarray:
    """ops::gemv over each row of x (batch x cols) -> batch x rows."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    batch = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((batch, rows), np.float32)
    _check(lib().orc_gemv_batch(quant, data.ctypes.data, data.nbytes, rows, cols, _fp(x), _fp(y), batch, threads),
           "gemv")
    return y[0] if x.ndim == 1 else y


def gemv_rows(quant: int, data: np.ndarray, rows: int, cols: int, x: np.ndarray, row0: int, row_end: int,
              threads: int = 1) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(row_end - row0, np.float32)
    _check(lib().orc_gemv_rows(quant, data.ctypes.data, data.nbytes, rows, cols, _fp(x), _fp(y), row0, row_end,
                               threads), "gemv_rows")
    return y


def expert_gemv(quant: int, data: np.ndarray, n_expert: int, rows: int, cols: int, e: int,
                x: np.ndarray) -> np.ndarray:
    """ops::expert_gemv for each row of x (batch x rows) -> batch x cols."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    xs = x.reshape(-1, rows)
    y = np.empty((xs.shape[0], cols), np.float32)
    for b in range(xs.shape[0]):
        xb = np.ascontiguousarray(xs[b])
        yb = np.empty(cols, np.float32)
        _check(lib().orc_expert_gemv(quant, data.ctypes.data, data.nbytes, n_expert, rows, cols, e, _fp(xb),
                                     _fp(yb)), "expert_gemv")
        y[b] = yb
    return y[0] if x.ndim == 1 else y


def _rows(x: np.ndarray, n: int) -> np.ndarray:
    return np.array(x, dtype=np.float32, copy=True).reshape(-1, n)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """ops::rms_norm (ops.rs:45-56) of every row of x (last axis = w's length)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = _rows(x, w.size)
    for r in out:
        lib().orc_rms_norm(_fp(r), _fp(w), w.size, eps)
    return out.reshape(np.shape(x))


def l2_norm(x: np.ndarray, head_dim: int, eps: float) -> np.ndarray:
    """ops::l2_norm (ops.rs:71-81) of every head_dim-long head of x."""
    out = _rows(x, head_dim)
    for r in out:
        lib().orc_l2_norm(_fp(r), head_dim, eps)
    return out.reshape(np.shape(x))


def softmax(x: np.ndarray, n: int) -> np.ndarray:
    """ops::softmax (ops.rs:107-119) of every n-long row of x."""
    out = _rows(x, n)
    for r in out:
        lib().orc_softmax(_fp(r), n)
    return out.reshape(np.shape(x))


def rope_neox(x: np.ndarray, head_dim: int, pos: int, n_rot: int, freq_base: float) -> np.ndarray:
    """ops::rope_neox (ops.rs:121-140) of every head_dim-long head of x at one position."""
    out = _rows(x, head_dim)
    for r in out:
        lib().orc_rope_neox(_fp(r), head_dim, pos, n_rot, head_dim, freq_base)
    return out.reshape(np.shape(x))


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """ops::add_into (ops.rs:164-168): a + b in f32."""
    out = np.array(a, dtype=np.float32, copy=True).reshape(-1)
    bb = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    lib().orc_add(_fp(out), _fp(bb), out.size)
    return out.reshape(np.shape(a))


def expf_misrounded(lo: float, hi: float, cap: int) -> np.ndarray:
    """Inputs in [lo, hi] where the C library's expf (the reference's f32::exp)
    is not the correctly rounded exp (test support)."""
    out = np.empty(cap, np.float32)
    n = lib().orc_expf_misrounded(lo, hi, _fp(out), cap)
    return out[:n].copy()


def expf_tie_pairs(lo: float, hi: float, cap: int) -> np.ndarray:
    """[n, 2] pairs x1 < x2 a few floats apart where expf ties and the
    correctly rounded exp does not (test support)."""
    out = np.empty((cap, 2), np.float32)
    n = lib().orc_expf_tie_pairs(lo, hi, _fp(out), cap)
    return out[:n].copy()


def route_logits(logits: np.ndarray, top_k: int) -> tuple[np.ndarray, np.ndarray]:
    """MoeLayer::route from the logits on (moe.rs:57-91) for each row."""
    lg = np.array(logits, dtype=np.float32, copy=True).reshape(-1, logits.shape[-1])
    ids = np.empty((lg.shape[0], top_k), np.int64)
    w = np.empty((lg.shape[0], top_k), np.float32)
    for t in range(lg.shape[0]):
        row = np.ascontiguousarray(lg[t])
        idt = np.empty(top_k, np.int64)
        wt = np.empty(top_k, np.float32)
        _check(lib().orc_moe_route_logits(_fp(row), row.size, top_k, idt.ctypes.data_as(C.POINTER(C.c_int64)),
                                          _fp(wt)), "route")
        ids[t], w[t] = idt, wt
    return ids, w


class MoeWeights(C.Structure):
    """orc_moe_weights (strata_oracle.h)."""
    _fields_ = []
    for nm in ["router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp", "down_shexp",
               "gate_inp_shexp"]:
        _fields_ += [(f"quant_{nm}", C.c_uint32), (nm, C.c_void_p), (f"{nm}_len", C.c_size_t)]
    _fields_ += [("n_embd", C.c_int64), ("n_expert", C.c_int64), ("top_k", C.c_int64), ("n_ff", C.c_int64),
                 ("n_ff_shexp", C.c_int64)]


def moe_layer(tensors: dict, n_embd: int, n_expert: int, top_k: int, n_ff: int, n_ff_shexp: int,
              x: np.ndarray, logits: np.ndarray | None, threads: int = 1):
    """MoeLayer route + combine for each token of x (tokens x n_embd).

    tensors maps name -> (quant, uint8 array); names as in MoeLayer
    (router optional when logits are given). Returns (out, ids, weights)."""
    keep = []
    L = MoeWeights()
    for nm in ["router", "gate_exps", "up_exps", "down_exps", "gate_shexp", "up_shexp", "down_shexp",
               "gate_inp_shexp"]:
        if nm in tensors:
            q, arr = tensors[nm]
            arr = np.ascontiguousarray(arr, dtype=np.uint8)
            keep.append(arr)
            setattr(L, f"quant_{nm}", q)
            setattr(L, nm, arr.ctypes.data)
            setattr(L, f"{nm}_len", arr.nbytes)
    L.n_embd, L.n_expert, L.top_k, L.n_ff, L.n_ff_shexp = n_embd, n_expert, top_k, n_ff, n_ff_shexp
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_embd)
    T = x.shape[0]
    out = np.empty((T, n_embd), np.float32)
    ids = np.empty((T, top_k), np.int64)
    w = np.empty((T, top_k), np.float32)
    lgp = None
    if logits is not None:
        lg = np.ascontiguousarray(logits, dtype=np.float32).reshape(T, n_expert)
        keep.append(lg)
        lgp = _fp(lg)
    _check(lib().orc_moe_layer(C.byref(L), _fp(x), lgp, T, _fp(out), ids.ctypes.data_as(C.POINTER(C.c_int64)),
                               _fp(w), threads), "moe_layer")
    return out, ids, w
