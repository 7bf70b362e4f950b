"""The Python mirror of ComputeBackend's elementwise methods
(crates/strata-core/src/backend.rs:37-50) without a GPU: CudaBackend's
in-place wrappers are driven through a stand-in context that computes with
the oracle, so the argument order, the RopeCfg fields and the in-place
writes are checked here; the device itself is checked in
tests/test_elementwise_gpu.py. Also the host-side length rules the reference
has: rms_norm needs a weight per value (ops::rms_norm indexes w[i]), add
works over the common length (ops::add_into zips)."""
import numpy as np
import pytest

import oracle
import strata_cuda as sc
from synth import rng


class OracleCtx:
    """Context's host-slice elementwise methods, computed by the oracle."""

    def rms_norm(self, x, w, eps):
        return oracle.rms_norm(np.asarray(x, np.float32).reshape(-1), np.asarray(w, np.float32).reshape(-1), eps)

    def l2_norm(self, head, eps):
        h = np.asarray(head, np.float32).reshape(-1)
        return oracle.l2_norm(h, h.size, eps)

    def softmax(self, xs):
        v = np.asarray(xs, np.float32).reshape(-1)
        return oracle.softmax(v, v.size)

    def rope_neox(self, head, pos, n_rot, head_dim, freq_base):
        return oracle.rope_neox(np.asarray(head, np.float32).reshape(-1), head_dim, pos, n_rot, freq_base)

    def add(self, a, b):
        a = np.asarray(a, np.float32).reshape(-1).copy()
        n = min(a.size, np.asarray(b).size)
        a[:n] = oracle.add(a[:n], np.asarray(b, np.float32).reshape(-1)[:n])
        return a


def backend():
    be = object.__new__(sc.CudaBackend)
    be.ctx, be._cache = OracleCtx(), {}
    return be


def test_elementwise_trait_methods_write_in_place():
    be, g = backend(), rng(77)
    x = g.standard_normal(64).astype(np.float32)
    w = g.standard_normal(64).astype(np.float32)
    y = x.copy()
    be.rms_norm(y, w, 1e-6)
    assert np.array_equal(y, oracle.rms_norm(x, w, 1e-6))
    h = x.copy()
    be.l2_norm(h, 0.0)
    assert np.array_equal(h, oracle.l2_norm(x, 64, 0.0))
    s = x.copy()
    be.softmax(s)
    assert np.array_equal(s, oracle.softmax(x, 64))
    r = x.copy()
    be.rope_neox(r, sc.RopeCfg(pos=17, n_rot=32, head_dim=64, freq_base=1e6))
    assert np.array_equal(r, oracle.rope_neox(x, 64, 17, 32, 1e6))
    a = x.copy()
    be.add(a, w[:40])
    assert np.array_equal(a[:40], x[:40] + w[:40]) and np.array_equal(a[40:], x[40:])


def test_length_rules_are_checked_before_the_device():
    ctx = object.__new__(sc.Context)
    ctx.h = None
    with pytest.raises(sc.BackendError) as ei:
        ctx.rms_norm(np.ones(8, np.float32), np.ones(7, np.float32), 0.0)
    assert ei.value.code == sc.ERR_INVALID
    a = np.arange(4, dtype=np.float32)
    assert np.array_equal(ctx.add(a, np.zeros(0, np.float32)), a)  # nothing in common: a unchanged


class CountingCtx:
    """A stand-in context that records uploads and frees (no device)."""

    def __init__(self):
        self.live = set()

    def upload(self, data, quant, rows, cols, n_expert=0):
        w = sc.Weight(self, object(), quant, n_expert, rows, cols)
        w.free = lambda w=w: self.live.discard(id(w))
        self.live.add(id(w))
        return w

    def gemv(self, w, x):
        return np.zeros(w.rows, np.float32)


def test_weight_cache_evicts_least_recently_used_over_budget():
    """gpu.rs:577-599 (a 24 MiB budget and three 10 MiB matrices: the first
    must go), with the LRU order of WeightCache (gpu.rs:61-112)."""
    be = object.__new__(sc.CudaBackend)
    be.ctx, be.budget, be._cache, be._bytes = CountingCtx(), 24 << 20, sc.OrderedDict(), 0
    cols = 4096
    rows = (10 << 20) // sc.byte_size(sc.Q8_0, cols)
    mats = [np.zeros(rows * sc.byte_size(sc.Q8_0, cols), np.uint8) for _ in range(3)]
    ts = [sc.QuantTensor(f"big{i}", sc.Q8_0, rows, cols, m) for i, m in enumerate(mats)]
    x, y = np.ones(cols, np.float32), np.empty(rows, np.float32)
    for t in ts:
        be.gemv(t, x, y)
    assert be.resident_bytes() <= 2 * mats[0].nbytes and len(be.ctx.live) == 2
    assert [k[0] for k in be._cache] == [mats[1].ctypes.data, mats[2].ctypes.data]  # big0 went first
    be.gemv(ts[1], x, y)       # big1 becomes the most recent
    be.gemv(ts[0], x, y)       # big0 comes back: big2, now the least recent, goes
    assert [k[0] for k in be._cache] == [mats[1].ctypes.data, mats[0].ctypes.data]
    assert be.resident_bytes() == 2 * mats[0].nbytes and len(be.ctx.live) == 2
