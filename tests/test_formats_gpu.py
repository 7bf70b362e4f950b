"""The block formats beyond the benchmark's four (Q4_0, Q4_1, Q5_0, Q5_1, Q8_1,
Q2_K, Q3_K, IQ4_NL, IQ4_XS, MXFP4, NVFP4, Q2_0) through the device paths.

Dequant against strata-gguf's dequantize_row (crates/strata-gguf/src/dequant.rs:
87-206, 304-445, restated in the oracle) bit for bit, including non-finite
fp16 scales (x86 NaN propagation); the reference's own known answers
(dequant_tests.rs:26-158) and its finite-on-LCG-bytes check (:186-244); the
GEMV and expert GEMV within rel_err 1e-3 of the oracle's f64-accumulated
ops::gemv / ops::expert_gemv.
"""
import numpy as np
import pytest

import oracle
import strata_cuda as sc
import synth
from conftest import rel_err
from golden import reference_cases as rc
from synth import activations, quant_matrix

pytestmark = pytest.mark.gpu
FORMATS = synth.OTHER_FORMATS
FP16_SCALED = [synth.Q4_0, synth.Q4_1, synth.Q5_0, synth.Q5_1, synth.Q8_1, synth.Q2_K, synth.IQ4_NL,
               synth.IQ4_XS, synth.Q2_0]


@pytest.fixture(scope="module")
def ctx():
    c = sc.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("quant", FORMATS)
def test_dequant_bit_exact(ctx, quant):
    bs, ts = synth.BLOCK[quant]
    rows, cols = 6, 4 * 256
    data = quant_matrix(700 + quant, quant, rows, cols).reshape(rows, -1)
    if quant in FP16_SCALED:
        # non-finite and extreme fp16 d in a few blocks: NaN payloads, inf, subnormal, max
        special = np.array([0x7E01, 0x7C00, 0xFC00, 0x0001, 0x7BFF, 0xFE55], np.uint16).view(np.uint8)
        per_row = cols // bs
        for i in range(6):
            blk = i % per_row
            data[i, ts * blk:ts * blk + 2] = special[2 * i:2 * i + 2]
    data = data.reshape(-1)
    w = ctx.upload(data, quant, rows, cols)
    got = ctx.dequant(w)
    want = oracle.dequantize(quant, data, rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), sc.NAMES[quant]
    w.free()


@pytest.mark.parametrize("case", [c for c in rc.KATS["dequant"] if c["quant"] in FORMATS], ids=lambda c: c["name"])
def test_reference_known_answers_on_gpu(ctx, case):
    b = rc.dequant_case(case)
    w = ctx.upload(b, case["quant"], 1, case["n"])
    out = ctx.dequant(w).reshape(-1)
    for j, v in case["expect"]:
        assert out[j] == v, (case["name"], j, out[j], v)
    w.free()


def test_reference_every_type_finite_on_lcg_bytes(ctx):
    spec = rc.KATS["finite_lcg"]
    for quant, n in spec["cases"]:
        if quant not in FORMATS:
            continue
        b = rc.lcg_block(quant, sc.byte_size(quant, n), spec)
        w = ctx.upload(b, quant, 1, n)
        out = ctx.dequant(w)
        assert np.isfinite(out).all(), sc.NAMES[quant]
        assert np.array_equal(out.view(np.uint32), oracle.dequantize(quant, b, 1, n).view(np.uint32))
        w.free()


@pytest.mark.parametrize("quant", FORMATS)
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_gemv(ctx, quant, batch):
    rows, cols = 96, 1024
    data = quant_matrix(800 + quant, quant, rows, cols)
    x = activations(801 + batch, batch, cols)
    w = ctx.upload(data, quant, rows, cols)
    got = ctx.gemv(w, x)
    want = oracle.gemv(quant, data, rows, cols, x, threads=4)
    for b in range(batch):
        assert rel_err(got.reshape(batch, rows)[b], want.reshape(batch, rows)[b]) < 1e-3, (sc.NAMES[quant], b)
    w.free()


@pytest.mark.parametrize("quant", [synth.Q4_0, synth.Q3_K, synth.IQ4_XS, synth.NVFP4])
def test_expert_gemv(ctx, quant):
    E, IN, OUT = 3, 128, 512
    data = quant_matrix(900 + quant, quant, IN, OUT, E)
    w = ctx.upload(data, quant, IN, OUT, n_expert=E)
    x = activations(901, 2, IN)
    for e in range(E):
        got = ctx.expert_gemv(w, e, x)
        for b in range(2):
            want = oracle.expert_gemv(quant, data, E, IN, OUT, e, x[b]).reshape(-1)
            assert rel_err(got[b], want) < 1e-3, (sc.NAMES[quant], e, b)
    w.free()


def test_q2_0_structural_invariant_on_gpu(ctx):
    """dequant_tests.rs:43-60 through the device: every value is -d, 0, +d or +2d."""
    w = ctx.upload(rc.q2_0_invariant_block(), synth.Q2_0, 1, 64)
    out = ctx.dequant(w).reshape(-1)
    d = 0.5
    assert all(min(abs(v + d), abs(v), abs(v - d), abs(v - 2 * d)) < 1e-6 for v in out)
    w.free()
