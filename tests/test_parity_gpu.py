"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Bars: dequant bit-exact with dequantize_row; GEMV / expert GEMV within
rel_err 1e-3 (fp32 accumulation) of ops::gemv / ops::expert_gemv, which
accumulate in f64 (crates/strata-core/src/ops.rs:14-28,169-195).
"""
import numpy as np
import pytest

import oracle
import strata_cuda as sc
from conftest import rel_err
from golden import reference_cases as rc
from synth import Q4K_SWEEP, Q4_K, Q5_K, Q6_K, Q8_0, F32, F16, BF16, activations, quant_blocks, quant_matrix, rng

pytestmark = pytest.mark.gpu
TOL = 1e-3
BS = {F32: 1, F16: 1, BF16: 1, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}


@pytest.fixture(scope="module")
def ctx():
    c = sc.Context(0)
    yield c
    c.close()


def _special_scales(blocks, quant):
    """Overwrite some fp16 scales with subnormal / inf / NaN / negative bit patterns."""
    specials = np.array([0x0001, 0x03FF, 0x7C00, 0xFC00, 0x7E01, 0xFD55, 0x8400, 0x0000], np.uint16)
    off = 208 if quant == Q6_K else 0
    for i, s in enumerate(specials):
        blocks[i, off:off + 2] = np.array([s], np.uint16).view(np.uint8)
        if quant in (Q4_K, Q5_K):
            blocks[i + 8, 2:4] = np.array([s], np.uint16).view(np.uint8)
    return blocks


@pytest.mark.parametrize("quant", [F16, BF16])
def test_every_16_bit_pattern(ctx, quant):
    """All 65,536 F16 / BF16 bit patterns through the device's conversion
    against the oracle's restatement of the `half` crate (the f16 -> f32 of
    crates/strata-gguf/src/dequant.rs:28-36): bit-exact for every finite value
    and both infinities; NaNs stay NaN (their payload bits are not pinned)."""
    data = np.arange(65536, dtype=np.uint16).view(np.uint8)
    w = ctx.upload(data, quant, 64, 1024)
    got = ctx.dequant(w).reshape(-1)
    want = oracle.dequantize(quant, data, 64, 1024).reshape(-1)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    assert nan.sum() == (2046 if quant == F16 else 254)
    w.free()


@pytest.mark.parametrize("case", [c for c in rc.KATS["dequant"] if c["quant"] in BS], ids=lambda c: c["name"])
def test_reference_dequant_known_answers_on_gpu(ctx, case):
    """The reference's dequant known answers for the benchmark and float types
    (dequant_tests.rs:70-79, :123-140, :160-169) through the device."""
    w = ctx.upload(rc.dequant_case(case), case["quant"], 1, case["n"])
    out = ctx.dequant(w).reshape(-1)
    for j, v in case["expect"]:
        assert out[j] == np.float32(v), (case["name"], j, out[j], v)
    w.free()


@pytest.mark.parametrize("quant", [Q8_0, Q4_K, Q5_K, Q6_K, F32, F16, BF16])
def test_dequant_bit_exact(ctx, quant):
    rows, cols = 24, 1024
    nb = rows * cols // BS[quant]
    blocks = quant_blocks(rng(500 + quant), quant, nb)
    if quant in (Q8_0, Q4_K, Q5_K, Q6_K):
        blocks = _special_scales(blocks, quant)
    data = blocks.reshape(-1)
    w = ctx.upload(data, quant, rows, cols)
    got = ctx.dequant(w)
    want = oracle.dequantize(quant, data, rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    part = ctx.dequant(w, row0=5, nrows=7)
    assert np.array_equal(part.view(np.uint32), want[5:12].view(np.uint32))
    w.free()


@pytest.mark.parametrize("quant", [Q8_0, Q4_K, Q5_K, Q6_K, F32, F16, BF16])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8])
def test_gemv_parity_small(ctx, quant, batch, threads):
    rows, cols = 301, 2048     # rows not a multiple of any row tile
    data = quant_matrix(600 + quant, quant, rows, cols)
    x = activations(700 + batch, batch, cols)
    w = ctx.upload(data, quant, rows, cols)
    got = ctx.gemv(w, x)
    want = oracle.gemv(quant, data, rows, cols, x, threads=threads)
    for b in range(batch):
        assert rel_err(got[b], want[b]) < TOL, (quant, batch, b)
    w.free()


@pytest.mark.parametrize("quant", [Q4_K, Q5_K, Q6_K, Q8_0])
def test_gemv_one_block_rows(ctx, quant, threads):
    # K = one block: the smallest row, every lane but a few idle
    cols = BS[quant]
    rows = 77
    data = quant_matrix(800 + quant, quant, rows, cols)
    x = activations(801, 3, cols)
    w = ctx.upload(data, quant, rows, cols)
    got = ctx.gemv(w, x)
    want = oracle.gemv(quant, data, rows, cols, x, threads=threads)
    assert rel_err(got, want) < TOL
    w.free()


@pytest.mark.parametrize("k,n", Q4K_SWEEP)
@pytest.mark.parametrize("batch", [1, 8])
def test_q4_k_sweep_shapes(ctx, k, n, batch, threads):
    data = quant_matrix(1000 + k + n, Q4_K, n, k)
    x = activations(1001, batch, k)
    w = ctx.upload(data, Q4_K, n, k)
    got = ctx.gemv(w, x)
    want = oracle.gemv(Q4_K, data, n, k, x, threads=threads)
    assert rel_err(got, want) < TOL
    w.free()


@pytest.mark.parametrize("k,n,batch", [(2048, 151936, 2), (2048, 151936, 4), (2304, 40000, 8)])
def test_gemv_large_result_in_slices(ctx, k, n, batch, threads):
    """A host-buffer result above 1 MiB is computed in row slices, each copied
    out while the next computes (K = 2304 has no tensor map: the bulk-copy
    form): every row against ops::gemv, and against the device-buffer entry
    point's result of the same product."""
    torch = pytest.importorskip("torch")
    data = quant_matrix(1050 + k + batch, Q4_K, n, k)
    x = activations(1051 + batch, batch, k)
    w = ctx.upload(data, Q4_K, n, k)
    got = ctx.gemv(w, x)
    want = oracle.gemv(Q4_K, data, n, k, x, threads=threads)
    assert rel_err(got, want) < TOL
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((batch, n), dtype=torch.float32, device="cuda")
    ctx.gemv_dev(w, xd.data_ptr(), yd.data_ptr(), batch)
    torch.cuda.synchronize()
    assert rel_err(got, yd.cpu().numpy()) < 1e-6
    again = ctx.gemv(w, x)
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))
    w.free()


def test_q8_0_config_shape(ctx, threads):
    data = quant_matrix(1100, Q8_0, 4096, 4096)
    x = activations(1101, 1, 4096)
    w = ctx.upload(data, Q8_0, 4096, 4096)
    assert rel_err(ctx.gemv(w, x), oracle.gemv(Q8_0, data, 4096, 4096, x, threads=threads)) < TOL
    w.free()


@pytest.mark.parametrize("case", rc.KATS["gemv"], ids=lambda c: c["name"])
def test_reference_gemv_cases_on_gpu(ctx, case):
    q, data, rows, cols, x = rc.gemv_case(case)
    w = ctx.upload(data, q, rows, cols)
    got = ctx.gemv(w, x)
    want = oracle.gemv(q, data, rows, cols, x)
    tol = case.get("abs_tol", 1e-6)
    assert np.max(np.abs(got.astype(np.float64) - want)) < tol
    w.free()


@pytest.mark.parametrize("quant", [Q4_K, Q5_K, Q6_K, Q8_0, F32, F16, BF16])
@pytest.mark.parametrize("batch", [1, 3, 6])
def test_expert_gemv_parity(ctx, quant, batch):
    E, IN, OUT = 3, 512, 1024 if quant != F32 else 40
    data = quant_matrix(1200 + quant, quant, IN, OUT, n_expert=E)
    x = activations(1201 + batch, batch, IN)
    w = ctx.upload(data, quant, IN, OUT, n_expert=E)
    for e in range(E):
        got = ctx.expert_gemv(w, e, x)
        want = oracle.expert_gemv(quant, data, E, IN, OUT, e, x)
        assert rel_err(got, want) < TOL, (quant, e)
    w.free()


@pytest.mark.parametrize("IN,OUT", [(2048, 512), (512, 2048)])
def test_expert_gemv_moe_shapes(ctx, IN, OUT):
    E = 4
    data = quant_matrix(1300 + IN, Q4_K, IN, OUT, n_expert=E)
    x = activations(1301, 2, IN)
    w = ctx.upload(data, Q4_K, IN, OUT, n_expert=E)
    for e in (0, E - 1):
        assert rel_err(ctx.expert_gemv(w, e, x), oracle.expert_gemv(Q4_K, data, E, IN, OUT, e, x)) < TOL
    w.free()


def test_reference_expert_case_on_gpu(ctx):
    q, data, E, rows, cols, x = rc.expert_case(rc.KATS["expert_gemv"][0])
    w = ctx.upload(data, q, rows, cols, n_expert=E)
    for e in range(E):
        got = ctx.expert_gemv(w, e, x)
        want = oracle.expert_gemv(q, data, E, rows, cols, e, x)
        assert np.max(np.abs(got - want)) < 1e-3
    w.free()


def test_backend_trait_mirror(ctx):
    be = sc.CudaBackend(0)
    assert be.name() == "cuda"
    data = quant_matrix(1400, Q4_K, 64, 512)
    t = sc.QuantTensor("blk.0.ffn_up.weight", Q4_K, 64, 512, data)
    x = activations(1401, 1, 512)[0]
    y = np.empty(64, np.float32)
    be.gemv(t, x, y, None)
    assert rel_err(y, oracle.gemv(Q4_K, data, 64, 512, x)) < TOL
    be.gemv(t, x, y, None)  # second call hits the resident copy
    assert len(be._cache) == 1
    be.close()


def test_backend_weight_cache_evicts_over_budget():
    """crates/strata-backend-wgpu/src/gpu.rs:577-599 on the device: a 24 MiB budget and three
    10 MiB matrices (Q8_0 here; F32 [n x 1] there): the first must go, and what stays
    resident is what the context holds."""
    be = sc.CudaBackend(0, budget_bytes=24 << 20)
    cols = 4096
    rows = (10 << 20) // sc.byte_size(Q8_0, cols)
    x = activations(1402, 1, cols)[0]
    y = np.empty(rows, np.float32)
    mats = [quant_matrix(1403 + i, Q8_0, rows, cols) for i in range(3)]
    for i, m in enumerate(mats):
        be.gemv(sc.QuantTensor(f"big{i}", Q8_0, rows, cols, m), x, y, None)
    assert be.resident_bytes() <= 2 * mats[0].nbytes
    assert be.ctx.resident_bytes() == be.resident_bytes()
    assert rel_err(y, oracle.gemv(Q8_0, mats[2], rows, cols, x, threads=4)) < TOL
    be.close()


# ---- error behaviour (host-side checks; nothing here faults the device)

def test_errors(ctx):
    data = quant_matrix(1500, Q4_K, 4, 256)
    with pytest.raises(sc.BackendError) as e:
        ctx.upload(data[:-1], Q4_K, 4, 256)
    assert e.value.code == sc.ERR_TRUNCATED
    with pytest.raises(sc.BackendError) as e:
        ctx.upload(data, Q4_K, 2, 200)
    assert e.value.code == sc.ERR_TRUNCATED
    with pytest.raises(sc.BackendError) as e:
        ctx.upload(data, 16, 4, 256)  # IQ2_XXS: not on this path (a grid-table i-quant)
    assert e.value.code == sc.ERR_UNSUPPORTED_QUANT
    w = ctx.upload(data, Q4_K, 4, 256)
    with pytest.raises(sc.BackendError) as e:
        ctx.gemv(w, np.zeros((9, 256), np.float32))
    assert e.value.code == sc.ERR_INVALID
    with pytest.raises(sc.BackendError) as e:
        ctx.expert_gemv(w, 0, np.zeros(4, np.float32))
    assert e.value.code == sc.ERR_INVALID
    with pytest.raises(sc.BackendError):
        ctx.dequant(w, row0=3, nrows=5)
    w.free()
    ew = ctx.upload(quant_matrix(1501, Q4_K, 8, 256, n_expert=2), Q4_K, 8, 256, n_expert=2)
    with pytest.raises(sc.BackendError) as e:
        ctx.expert_gemv(ew, 2, np.zeros(8, np.float32))
    assert e.value.code == sc.ERR_INVALID
    ew.free()


def test_weight_budget(ctx):
    c = sc.Context(0)
    c.set_weight_budget(1 << 20)
    a = c.upload(quant_matrix(1600, Q4_K, 1024, 512), Q4_K, 1024, 512)  # 294,912 B
    assert c.resident_bytes() == 1024 * 288
    with pytest.raises(sc.BackendError) as e:
        c.upload(quant_matrix(1601, Q4_K, 4096, 512), Q4_K, 4096, 512)
    assert e.value.code == sc.ERR_BUDGET
    a.free()
    assert c.resident_bytes() == 0
    c.close()


def test_bounded_wait_times_out_and_recovers():
    """A wait shorter than the queued work returns STRATA_ERR_TIMEOUT; the work
    finishes normally and the context keeps working."""
    c = sc.Context(0)
    n, k = 151936, 2048
    data = quant_matrix(1700, Q4_K, n, k)
    w = c.upload(data, Q4_K, n, k)
    import torch
    x = torch.randn(8, k, device="cuda")
    y = torch.empty(8, n, device="cuda")
    torch.cuda.synchronize()
    for _ in range(200):
        c.gemv_dev(w, x.data_ptr(), y.data_ptr(), 8)
    c.set_wait_timeout_ms(1)
    with pytest.raises(sc.BackendError) as e:
        c.synchronize()
    assert e.value.code == sc.ERR_TIMEOUT
    c.set_wait_timeout_ms(60000)
    c.synchronize()
    xs = activations(1701, 1, k)
    assert rel_err(c.gemv(w, xs), oracle.gemv(Q4_K, data, n, k, xs, threads=8)) < TOL
    w.free()
    c.close()


# ---- the two decode kernel families (tensor-core and CUDA-core) on the same inputs

@pytest.mark.parametrize("path", [sc.Context.GEMV_CUDA_CORES, sc.Context.GEMV_TENSOR_CORES])
@pytest.mark.parametrize("quant", [Q4_K, Q5_K])
@pytest.mark.parametrize("batch", [1, 2, 4, 5, 8])
@pytest.mark.parametrize("rows,cols", [(203, 2048), (1000, 256), (64, 12288)])
def test_gemv_both_paths(quant, batch, rows, cols, path, threads):
    c = sc.Context(0)
    c.set_gemv_path(path)
    data = quant_matrix(2000 + quant + cols, quant, rows, cols)
    x = activations(2001 + batch, batch, cols)
    w = c.upload(data, quant, rows, cols)
    got = c.gemv(w, x)
    want = oracle.gemv(quant, data, rows, cols, x, threads=threads)
    assert rel_err(got, want) < TOL
    w.free()
    c.close()


@pytest.mark.parametrize("scale", [1e-30, 1e-6, 1.0, 1e4, 1e30])
def test_gemv_activation_magnitudes(ctx, scale, threads):
    """fp16 activation limbs carry a per-(column, block) power-of-two scale:
    tiny, huge, zero and mixed-magnitude activations stay within tolerance."""
    rows, cols = 96, 4096
    data = quant_matrix(2100, Q4_K, rows, cols)
    x = activations(2101, 3, cols) * np.float32(scale)
    x[1, :512] = 0.0                                   # an all-zero block
    x[2, ::7] *= np.float32(1e-3)                      # mixed magnitudes in one block
    w = ctx.upload(data, Q4_K, rows, cols)
    got = ctx.gemv(w, x.astype(np.float32))
    want = oracle.gemv(Q4_K, data, rows, cols, x.astype(np.float32), threads=threads)
    for b in range(3):
        assert rel_err(got[b], want[b]) < TOL, (scale, b)
    w.free()


def test_tensor_core_path_rejects_other_types():
    c = sc.Context(0)
    c.set_gemv_path(sc.Context.GEMV_TENSOR_CORES)
    w = c.upload(quant_matrix(2200, Q6_K, 8, 256), Q6_K, 8, 256)
    with pytest.raises(sc.BackendError) as e:
        c.gemv(w, np.zeros(256, np.float32))
    assert e.value.code == sc.ERR_UNSUPPORTED_QUANT
    w.free()
    c.close()


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (301, 2048), (77, 1024)])
def test_q8_0_bulk_kernel_equals_the_cuda_core_kernel(ctx, rows, cols, threads):
    """Q8_0 at batch 1-2 with K a multiple of 1024 runs the bulk-copy kernel;
    batch 3 still runs the CUDA-core kernel. Both do the same arithmetic in the
    same order, so each token's outputs agree bit for bit (and with ops::gemv
    within tolerance)."""
    data = quant_matrix(2500 + cols, Q8_0, rows, cols)
    x = activations(2501 + rows, 3, cols)
    w = ctx.upload(data, Q8_0, rows, cols)
    y3 = ctx.gemv(w, x)
    y1 = ctx.gemv(w, x[:1])
    y2 = ctx.gemv(w, x[:2])
    assert np.array_equal(y1[0].view(np.uint32), y3[0].view(np.uint32))
    assert np.array_equal(y2.view(np.uint32), y3[:2].view(np.uint32))
    assert rel_err(y1[0], oracle.gemv(Q8_0, data, rows, cols, x[:1], threads=threads)[0]) < TOL
    w.free()
