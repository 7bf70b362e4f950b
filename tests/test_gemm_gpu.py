"""Parity of the tensor-core prefill GEMM (through the C ABI) with the CPU oracle.

The reference runs prefill as one ops::gemv per prompt token
(crates/strata-core/src/generate.rs:116-118, crates/strata-core/src/ops.rs:14-28),
accumulating in f64. The GEMM stages activations as bf16, so the oracle is
ops::gemv on the bf16-rounded activations, and the bar is rel_err 1e-2
(the bf16-staged tolerance).
"""
import numpy as np
import pytest

import oracle
import strata_cuda as sc
from conftest import rel_err
from synth import Q4_K, Q5_K, Q6_K, Q8_0, F32, activations, bf16_bits, bf16_round, quant_matrix

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module")
def ctx():
    c = sc.Context(0)
    yield c
    c.close()


def _x(seed, m, k):
    x = activations(seed, m, k)
    return bf16_bits(x), bf16_round(x)


# (rows N, cols K, tokens M): ragged N and M, one and several token tiles,
# the 64/128/256 token-tile kernels, and a split-K case (few tiles, deep K)
SHAPES = [(256, 1024, 64), (301, 512, 5), (384, 2048, 130), (200, 768, 300), (256, 4096, 64), (128, 256, 1),
          (520, 1536, 257)]
# Q6_K rows (210-byte blocks) have a 16-byte pitch only when cols is a multiple of 2048
SHAPES_Q6 = [(256, 2048, 64), (301, 2048, 5), (384, 2048, 130), (200, 2048, 300), (256, 4096, 64), (128, 2048, 1),
             (520, 4096, 257)]
CASES = [(q, s) for q in (Q4_K, Q5_K) for s in SHAPES] + [(Q6_K, s) for s in SHAPES_Q6]


@pytest.mark.parametrize("quant,shape", CASES)
def test_gemm_parity(ctx, quant, shape, threads):
    rows, cols, m = shape
    data = quant_matrix(900 + quant + rows, quant, rows, cols)
    bits, xr = _x(901 + m, m, cols)
    w = ctx.upload(data, quant, rows, cols)
    got = ctx.gemm_bf16(w, bits)
    want = oracle.gemv(quant, data, rows, cols, xr, threads=threads)
    want = want.reshape(m, rows)
    errs = [rel_err(got[t], want[t]) for t in range(m)]
    assert max(errs) < TOL, (quant, shape, max(errs))
    w.free()


@pytest.mark.parametrize("quant", [Q5_K, Q6_K])
def test_gemm_f32_entry_rounds_to_bf16(ctx, quant):
    rows, cols, m = 256, 2048, 70
    data = quant_matrix(910 + quant, quant, rows, cols)
    x = activations(911, m, cols)
    w = ctx.upload(data, quant, rows, cols)
    a = ctx.gemm_f32(w, x)
    b = ctx.gemm_bf16(w, bf16_bits(x))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    w.free()


def test_gemm_deterministic(ctx):
    rows, cols, m = 256, 4096, 64        # split-K path
    data = quant_matrix(920, Q6_K, rows, cols)
    bits, _ = _x(921, m, cols)
    w = ctx.upload(data, Q6_K, rows, cols)
    a = ctx.gemm_bf16(w, bits)
    b = ctx.gemm_bf16(w, bits)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    w.free()


def test_gemm_single_term_is_coarser(ctx, threads):
    # one bf16 copy of the weights misses the bound the two-term staging meets
    rows, cols, m = 256, 4096, 8
    data = quant_matrix(930, Q5_K, rows, cols)
    bits, xr = _x(931, m, cols)
    w = ctx.upload(data, Q5_K, rows, cols)
    want = oracle.gemv(Q5_K, data, rows, cols, xr, threads=threads)
    ctx.set_gemm_terms(1)
    try:
        one = ctx.gemm_bf16(w, bits)
    finally:
        ctx.set_gemm_terms(2)
    two = ctx.gemm_bf16(w, bits)
    e1 = max(rel_err(one[t], want[t]) for t in range(m))
    e2 = max(rel_err(two[t], want[t]) for t in range(m))
    assert e2 < TOL and e1 > 5 * e2, (e1, e2)
    w.free()


def _rel_err_rows(y, ref):
    """rel_err of every row of y against the same row of ref (vectorised)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    floor = 1e-3 * np.maximum(np.max(np.abs(ref), axis=1, keepdims=True), 1e-30)
    return np.max(np.abs(y - ref) / np.maximum(np.abs(ref), floor), axis=1)


@pytest.mark.parametrize("quant,K,N,m", [(q, K, N, m) for (q, K, N) in [(Q5_K, 4096, 12288), (Q6_K, 4096, 12288),
                                                                        (Q5_K, 12288, 4096), (Q6_K, 12288, 4096)]
                                          for m in (64, 512, 2048)]
                         + [(Q4_K, 8192, 28672, 1024), (Q4_K, 28672, 8192, 1024)])
def test_gemm_config_shapes(ctx, quant, K, N, m, threads):
    """The mixed K-quant prefill configuration at full size, and the
    row-sharded projection configuration's two matrices. Every output is
    checked against an f64 product of the oracle's bit-exact dequantized
    weights with the bf16 activations (computed on the GPU in float64, where
    the sequential f64 sum of ops::gemv would take the CPU minutes), and
    sampled tokens x row ranges against ops::gemv itself."""
    torch = pytest.importorskip("torch")
    data = quant_matrix(940 + quant, quant, N, K)
    bits, xr = _x(941 + m, m, K)
    w = ctx.upload(data, quant, N, K)
    got = ctx.gemm_bf16(w, bits)
    assert np.isfinite(got).all()
    W = torch.from_numpy(oracle.dequantize(quant, data, N, K)).cuda().double()
    ref = (torch.from_numpy(xr).cuda().double() @ W.T).cpu().numpy()
    del W
    errs = _rel_err_rows(got, ref)
    assert errs.max() < TOL, (float(errs.max()), float(np.median(errs)))
    g = np.random.default_rng(942 + m)
    toks = sorted(set([0, m - 1] + list(g.integers(0, m, 2))))
    for t in toks:
        for r0 in (0, N - 256, int(g.integers(0, N - 256))):
            want = oracle.gemv_rows(quant, data, N, K, xr[t], r0, r0 + 256, threads=threads)
            assert rel_err(got[t, r0:r0 + 256], want) < TOL, (t, r0)
            assert rel_err(ref[t, r0:r0 + 256], want) < 1e-6, (t, r0)
    w.free()


def test_gemm_rejects(ctx):
    data = quant_matrix(950, Q8_0, 64, 256)
    w = ctx.upload(data, Q8_0, 64, 256)
    with pytest.raises(sc.BackendError) as e:
        ctx.gemm_bf16(w, np.zeros((4, 256), np.uint16))
    assert e.value.code == sc.ERR_UNSUPPORTED_QUANT
    w.free()
    wf = ctx.upload(np.zeros(64 * 256 * 4, np.uint8), F32, 64, 256)
    with pytest.raises(sc.BackendError) as e:
        ctx.gemm_bf16(wf, np.zeros((4, 256), np.uint16))
    assert e.value.code == sc.ERR_UNSUPPORTED_QUANT
    wf.free()
    # Q6_K rows of three super-blocks are 630 bytes: not a 16-byte row pitch
    d6 = quant_matrix(951, Q6_K, 16, 768)
    w6 = ctx.upload(d6, Q6_K, 16, 768)
    with pytest.raises(sc.BackendError) as e:
        ctx.gemm_bf16(w6, np.zeros((4, 768), np.uint16))
    assert e.value.code == sc.ERR_INVALID
    w6.free()


def test_gemm_dev_on_torch_stream(ctx):
    torch = pytest.importorskip("torch")
    rows, cols, m = 384, 2048, 96
    data = quant_matrix(960, Q4_K, rows, cols)
    bits, _ = _x(961, m, cols)
    w = ctx.upload(data, Q4_K, rows, cols)
    host = ctx.gemm_bf16(w, bits)
    xd = torch.from_numpy(bits.view(np.int16)).cuda()
    yd = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ctx.gemm_bf16_dev(w, xd.data_ptr(), yd.data_ptr(), m, s.cuda_stream)
    s.synchronize()
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), host.view(np.uint32))
    w.free()
