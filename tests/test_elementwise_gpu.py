"""The elementwise trait methods on the device against the CPU oracle.

ComputeBackend::rms_norm / l2_norm / softmax / rope_neox / add
(crates/strata-core/src/backend.rs:37-50) as CpuBackend runs them
(crates/strata-backend-cpu/src/lib.rs:44-67, ops.rs:45-168). The device forms
keep the reference's f64 arithmetic, so the f32 results are expected to be
the same bits, except where a CTA-order f64 sum or a libm-vs-CUDA f64
function lands within 1e-16 of an f32 rounding boundary: at most one ulp,
and rare. softmax's f32 exp is the C library's expf bit for bit on the max-shifted
domain (expf_libm, checked on every float of it at build time), so softmax
differs only where the device's CTA-order f64 sum does: at most two ulps with
the division; rows whose sum is exact in any order are the same bits. `add`
is exact.
"""
import numpy as np
import pytest

import oracle
import strata_cuda as sc
from synth import rng

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = sc.Context(0)
    yield c
    c.close()


def ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in units in the last place of f32 (same-sign finite values)."""
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


def assert_close(got, want, what, max_ulps=1):
    d = ulps(got, want)
    assert d.max() <= max_ulps, (what, int(d.max()))
    assert np.mean(d == 0) >= 0.999, (what, float(np.mean(d == 0)))


def test_reference_known_values(ctx):
    """ops_tests.rs:80-134 through the device."""
    s = 2.0 / np.sqrt(12.5)
    x = ctx.rms_norm(np.array([3.0, 4.0], np.float32), np.array([2.0, 2.0], np.float32), 0.0)
    assert abs(x[0] - np.float32(3.0 * s)) < 1e-6 and abs(x[1] - np.float32(4.0 * s)) < 1e-6
    h = ctx.l2_norm(np.array([3.0, 4.0, 0.0], np.float32), 0.0)
    assert abs(float(np.sqrt(np.sum(h * h))) - 1.0) < 1e-6
    r = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    assert np.array_equal(ctx.rope_neox(r, 0, 4, 4, 1e7), r)
    r = ctx.rope_neox(np.array([1.0, 0.0], np.float32), 1, 2, 2, 1.0)
    assert abs(r[0] - np.float32(np.cos(1.0))) < 1e-6 and abs(r[1] - np.float32(np.sin(1.0))) < 1e-6
    p = ctx.softmax(np.array([1.0, 2.0, 3.0, 0.5], np.float32))
    assert abs(float(np.sum(p.astype(np.float64))) - 1.0) < 1e-6 and p[2] > p[1] > p[0] > p[3]


@pytest.mark.parametrize("n", [1, 2, 7, 128, 2048, 5000])
def test_rms_norm_and_l2_norm(ctx, n):
    g = rng(100 + n)
    x = g.standard_normal(n).astype(np.float32) * 3
    w = g.standard_normal(n).astype(np.float32)
    for eps in (0.0, 1e-6):
        assert_close(ctx.rms_norm(x, w, eps), oracle.rms_norm(x, w, eps), ("rms_norm", n, eps))
        assert_close(ctx.l2_norm(x, eps), oracle.l2_norm(x, n, eps), ("l2_norm", n, eps))


@pytest.mark.parametrize("n", [1, 3, 256, 2048, 151936])
def test_softmax(ctx, n):
    x = (rng(200 + n).standard_normal(n) * 4).astype(np.float32)
    assert_close(ctx.softmax(x), oracle.softmax(x, n), ("softmax", n), max_ulps=2)


def test_softmax_exp_is_the_c_librarys_expf(ctx):
    """f32::exp is the C library's expf, which is not correctly rounded: the
    device matches it bit for bit (expf_libm). Rows of one 0 (the maximum, so
    the exp arguments are the values themselves) and 255 inputs where expf
    differs from the correctly rounded exp, all in [-8, 0]: every exp is then
    above 3.4e-4, so the f64 sum of the row is exact in any order and the
    outputs must be the same bits."""
    m = oracle.expf_misrounded(-8.0, -0.25, 8 * 255)
    assert m.size == 8 * 255
    x = np.zeros((8, 256), np.float32)
    x[:, 1:] = rng(250).permutation(m).reshape(8, 255)
    got = np.stack([ctx.softmax(r) for r in x])
    want = oracle.softmax(x, 256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), int(ulps(got, want).max())


@pytest.mark.parametrize("head_dim,n_rot,pos,base", [(128, 128, 1234, 1e6), (128, 64, 7, 1e4), (64, 64, 0, 1e7),
                                                     (80, 33, 99, 5e5), (32, 200, 3, 1e4), (2, 2, 1, 1.0)])
def test_rope_neox(ctx, head_dim, n_rot, pos, base):
    x = rng(300 + head_dim + n_rot).standard_normal(head_dim).astype(np.float32)
    want = oracle.rope_neox(x, head_dim, pos, n_rot, base)
    assert_close(ctx.rope_neox(x, pos, n_rot, head_dim, base), want, ("rope", head_dim, n_rot, pos))


def test_add_is_exact(ctx):
    g = rng(400)
    a = g.standard_normal(4099).astype(np.float32)
    b = g.standard_normal(4099).astype(np.float32)
    assert np.array_equal(ctx.add(a, b), oracle.add(a, b))


def test_device_forms_many_rows(ctx):
    import torch
    g = rng(500)
    rows, n = 7, 2048
    x = g.standard_normal((rows, n)).astype(np.float32)
    w = g.standard_normal(n).astype(np.float32)
    st = torch.cuda.Stream()
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    st.wait_stream(torch.cuda.current_stream())
    ctx.rms_norm_dev(xd.data_ptr(), wd.data_ptr(), n, rows, 1e-6, st.cuda_stream)
    st.synchronize()
    assert_close(xd.cpu().numpy(), oracle.rms_norm(x, w, 1e-6), "rms_norm_dev")

    heads, hd = 32, 128
    q = g.standard_normal((heads, hd)).astype(np.float32)
    qd = torch.from_numpy(q).cuda()
    st.wait_stream(torch.cuda.current_stream())
    ctx.rope_neox_dev(qd.data_ptr(), hd, heads, 64, 4321, 1e6, st.cuda_stream)
    st.synchronize()
    assert_close(qd.cpu().numpy(), oracle.rope_neox(q, hd, 4321, 64, 1e6), "rope_neox_dev")
    qd2 = torch.from_numpy(q).cuda()
    st.wait_stream(torch.cuda.current_stream())
    ctx.l2_norm_dev(qd2.data_ptr(), hd, heads, 1e-6, st.cuda_stream)
    st.synchronize()
    assert_close(qd2.cpu().numpy(), oracle.l2_norm(q, hd, 1e-6), "l2_norm_dev")

    s = (g.standard_normal((5, 151936)) * 3).astype(np.float32)
    sd = torch.from_numpy(s).cuda()
    st.wait_stream(torch.cuda.current_stream())
    ctx.softmax_dev(sd.data_ptr(), 151936, 5, st.cuda_stream)
    st.synchronize()
    assert_close(sd.cpu().numpy(), oracle.softmax(s, 151936), "softmax_dev", max_ulps=2)

    a = torch.from_numpy(x.reshape(-1).copy()).cuda()
    b = torch.from_numpy(np.tile(w, rows)).cuda()
    st.wait_stream(torch.cuda.current_stream())
    ctx.add_dev(a.data_ptr(), b.data_ptr(), rows * n, st.cuda_stream)
    st.synchronize()
    assert np.array_equal(a.cpu().numpy(), oracle.add(x.reshape(-1), np.tile(w, rows))), "add_dev"


def test_rejects_bad_shapes(ctx):
    with pytest.raises(sc.BackendError):
        ctx.softmax(np.zeros(0, np.float32))


def test_backend_trait_methods_in_place():
    """CudaBackend's rms_norm / rope_neox / softmax / l2_norm / add write the
    caller's slices in place, as the trait's &mut [f32] arguments do."""
    be = sc.CudaBackend(0)
    g = rng(600)
    x = g.standard_normal(256).astype(np.float32)
    w = g.standard_normal(256).astype(np.float32)
    y = x.copy()
    be.rms_norm(y, w, 1e-6)
    assert_close(y, oracle.rms_norm(x, w, 1e-6), "trait rms_norm")
    r = x[:128].copy()
    be.rope_neox(r, sc.RopeCfg(pos=99, n_rot=64, head_dim=128, freq_base=1e6))
    assert_close(r, oracle.rope_neox(x[:128], 128, 99, 64, 1e6), "trait rope_neox")
    s = x.copy()
    be.softmax(s)
    assert_close(s, oracle.softmax(x, 256), "trait softmax", max_ulps=2)
    h = x[:128].copy()
    be.l2_norm(h, 0.0)
    assert_close(h, oracle.l2_norm(x[:128], 128, 0.0), "trait l2_norm")
    a = x.copy()
    be.add(a, w[:100])
    assert np.array_equal(a[:100], oracle.add(x[:100], w[:100])) and np.array_equal(a[100:], x[100:])
    be.close()
