"""The oracle's MoE layer pinned by an independent restatement.

strata-rs's own tests do not pin MoeLayer::route / combine numerically (only
their determinism on F32 weights), so the oracle's C restatement
(orc_moe_layer) is checked here against a second one written in numpy
straight from crates/strata-core/src/moe.rs:48-144 and ops.rs:85-92:

- route: logits from the router gemv on the bf16-rounded input; max-shifted
  exp in f32 (the system libm's expf, as Rust's f32::exp calls it), an f64
  sum, the f32 reciprocal `(1 / sum) as f32`, top-k by probability then
  lower id, ids ascending, weights divided in f64 by max(sum, 2^-14);
- combine: for each chosen expert in ascending id with a non-zero weight,
  silu(gate) * up -> down, `out += w * down` in f32; then the shared expert,
  scaled by sigmoid(gate_inp_shexp x).

The matrix products use the oracle's gemv / expert_gemv, which the
reference's known answers pin on their own. Ids and every output must agree
bit for bit.
"""
import ctypes
import ctypes.util

import numpy as np

import oracle
from synth import Q4_K, Q5_K, activations, bf16_round, quant_matrix

_libm = ctypes.CDLL(ctypes.util.find_library("m"))
_libm.expf.restype, _libm.expf.argtypes = ctypes.c_float, [ctypes.c_float]


def expf(v: np.ndarray) -> np.ndarray:
    return np.array([_libm.expf(float(a)) for a in np.asarray(v, np.float32).reshape(-1)], np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    return (x / (np.float32(1.0) + expf(-x))).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + expf(-x))).astype(np.float32)


def route(logits: np.ndarray, top_k: int):
    lg = np.asarray(logits, np.float32)
    mx = np.float32(lg.max())
    p = expf((lg - mx).astype(np.float32))
    s = 0.0
    for v in p:  # sequential f64 sum, in expert order
        s += float(v)
    inv = np.float32(1.0 / s)
    p = (p * inv).astype(np.float32)
    order = sorted(range(lg.size), key=lambda i: (-float(p[i]), i))[:top_k]
    ids = sorted(order)
    ws = 0.0
    for i in ids:
        ws += float(p[i])
    den = max(ws, 2.0 ** -14)
    return np.array(ids, np.int64), np.array([np.float32(float(p[i]) / den) for i in ids], np.float32)


def combine(t, dims, x, ids, w):
    E, n_embd, n_ff, n_ffs = dims["E"], dims["n_embd"], dims["n_ff"], dims["n_ff_s"]
    out = np.zeros(n_embd, np.float32)
    for e, we in zip(ids, w):
        if we == 0.0:
            continue
        g = oracle.expert_gemv(t["gate_exps"][0], t["gate_exps"][1], E, n_embd, n_ff, int(e), x).reshape(-1)
        u = oracle.expert_gemv(t["up_exps"][0], t["up_exps"][1], E, n_embd, n_ff, int(e), x).reshape(-1)
        h = (silu(g) * u).astype(np.float32)
        d = oracle.expert_gemv(t["down_exps"][0], t["down_exps"][1], E, n_ff, n_embd, int(e), h).reshape(-1)
        out = (out + (np.float32(we) * d).astype(np.float32)).astype(np.float32)
    g = oracle.gemv(t["gate_shexp"][0], t["gate_shexp"][1], n_ffs, n_embd, x).reshape(-1)
    u = oracle.gemv(t["up_shexp"][0], t["up_shexp"][1], n_ffs, n_embd, x).reshape(-1)
    h = (silu(g) * u).astype(np.float32)
    d = oracle.gemv(t["down_shexp"][0], t["down_shexp"][1], n_embd, n_ffs, h).reshape(-1)
    sg = sigmoid(oracle.gemv(t["gate_inp_shexp"][0], t["gate_inp_shexp"][1], 1, n_embd, x).reshape(-1))[0]
    return (out + (sg * d).astype(np.float32)).astype(np.float32)


def test_oracle_moe_layer_matches_a_numpy_restatement():
    dims = {"E": 16, "n_embd": 256, "n_ff": 256, "n_ff_s": 256}
    top_k = 4
    for qe, seed in ((Q4_K, 5100), (Q5_K, 5200)):
        t = {"router": (Q4_K, quant_matrix(seed, Q4_K, dims["E"], dims["n_embd"])),
             "gate_exps": (qe, quant_matrix(seed + 1, qe, dims["n_embd"], dims["n_ff"], dims["E"])),
             "up_exps": (qe, quant_matrix(seed + 2, qe, dims["n_embd"], dims["n_ff"], dims["E"])),
             "down_exps": (qe, quant_matrix(seed + 3, qe, dims["n_ff"], dims["n_embd"], dims["E"])),
             "gate_shexp": (Q4_K, quant_matrix(seed + 4, Q4_K, dims["n_ff_s"], dims["n_embd"])),
             "up_shexp": (Q4_K, quant_matrix(seed + 5, Q4_K, dims["n_ff_s"], dims["n_embd"])),
             "down_shexp": (Q4_K, quant_matrix(seed + 6, Q4_K, dims["n_embd"], dims["n_ff_s"])),
             "gate_inp_shexp": (Q4_K, quant_matrix(seed + 7, Q4_K, 1, dims["n_embd"]))}
        x = activations(seed + 8, 3, dims["n_embd"])
        out, ids, w = oracle.moe_layer(t, dims["n_embd"], dims["E"], top_k, dims["n_ff"], dims["n_ff_s"], x, None)
        for k in range(3):
            logits = oracle.gemv(Q4_K, t["router"][1], dims["E"], dims["n_embd"], bf16_round(x[k])).reshape(-1)
            rid, rw = route(logits, top_k)
            assert np.array_equal(rid, ids[k]), (k, rid, ids[k])
            assert np.array_equal(rw.view(np.uint32), w[k].view(np.uint32)), (k, rw, w[k])
            want = combine(t, dims, x[k], rid, rw)
            assert np.array_equal(want.view(np.uint32), out[k].view(np.uint32)), (qe, k)


def test_route_restatement_edge_cases():
    """Ties go to the lower id; a zero-sum guard of 2^-14; top_k = n_expert."""
    ids, w = route(np.zeros(8, np.float32), 3)
    assert list(ids) == [0, 1, 2]
    oids, ow = oracle.route_logits(np.zeros((1, 8), np.float32), 3)
    assert np.array_equal(ids, oids[0]) and np.array_equal(w.view(np.uint32), ow[0].view(np.uint32))
    lg = np.array([-200.0, 0.0, -200.0, -200.0], np.float32)  # three weights underflow to 0 after exp
    ids, w = route(lg, 4)
    oids, ow = oracle.route_logits(lg[None], 4)
    assert np.array_equal(ids, oids[0]) and np.array_equal(w.view(np.uint32), ow[0].view(np.uint32))
