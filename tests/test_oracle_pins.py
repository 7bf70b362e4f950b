"""Pins the CPU oracle (oracle/liboracle.so) before anything is compared with it.

* The reference's own known-answer tests (tests/golden/reference_kats.json).
* A second, vectorised numpy restatement of every block format, bit for bit
  (the reference pins Q4_K and Q5_K by no test of its own).
* The scalar codecs the `half` crate provides (f16 -> f32 over all 65,536
  patterns; bf16 round-to-nearest-even against numpy).
* Routing invariants of MoeLayer::route (crates/strata-core/src/moe.rs:48-92).
"""
import numpy as np
import pytest

import oracle
import numpy_dequant
from golden import reference_cases as rc
import synth
from synth import bf16_bits, quant_blocks, rng, Q4_K, Q5_K, Q6_K, Q8_0


@pytest.mark.parametrize("case", rc.KATS["dequant"], ids=lambda c: c["name"])
def test_reference_dequant_known_answers(case):
    out = oracle.dequantize_row(case["quant"], rc.dequant_case(case), case["n"])
    for idx, want in case["expect"]:
        assert out[idx] == np.float32(want)


@pytest.mark.parametrize("quant,n", [tuple(c) for c in rc.KATS["finite_lcg"]["cases"]])
def test_reference_every_type_finite_on_lcg_bytes(quant, n):
    nbytes = int(oracle.lib().orc_byte_size(quant, n))
    block = rc.lcg_block(quant, nbytes, rc.KATS["finite_lcg"])
    out = oracle.dequantize_row(quant, block, n)
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("case", rc.KATS["gemv"], ids=lambda c: c["name"])
def test_reference_gemv_known_answers(case):
    q, w, rows, cols, x = rc.gemv_case(case)
    y = oracle.gemv(q, w, rows, cols, x)
    deq = oracle.dequantize(q, w, rows, cols).astype(np.float64)
    expect = deq @ x.astype(np.float64)
    if case.get("exact"):
        assert y[0] == np.float32(deq[0, 0] * 1.0 - 2.0)
    else:
        assert np.max(np.abs(y.astype(np.float64) - expect)) < case["abs_tol"]


def test_reference_q8_0_gemv_value():
    # ops_tests.rs:55-58: expect = sum_j ((j % 7 - 3) * 0.5) * x[j] in f64
    case = rc.KATS["gemv"][0]
    q, w, rows, cols, x = rc.gemv_case(case)
    y = oracle.gemv(q, w, rows, cols, x)
    expect = sum(float((j % 7) - 3) * 0.5 * float(x[j]) for j in range(32))
    assert abs(float(y[0]) - expect) < 1e-4


@pytest.mark.parametrize("quant", [Q8_0, Q4_K, Q5_K, Q6_K])
def test_oracle_matches_independent_numpy_restatement(quant):
    g = rng(100 + quant)
    blocks = quant_blocks(g, quant, 512)
    # also cover extreme scales: subnormal, max and negative fp16 d / dmin
    extremes = np.array([0x0001, 0x03FF, 0x7BFF, 0xFBFF, 0x8001, 0x3C00], np.uint16).view(np.uint8)
    off = 208 if quant == Q6_K else 0
    for i in range(6):
        blocks[i, off:off + 2] = extremes[2 * i:2 * i + 2]
        if quant in (Q4_K, Q5_K):
            blocks[i, 2:4] = extremes[2 * ((i + 1) % 6):2 * ((i + 1) % 6) + 2]
    bs = 32 if quant == Q8_0 else 256
    got = oracle.dequantize_row(quant, blocks.reshape(-1), blocks.shape[0] * bs)
    want = numpy_dequant.DEQUANT[quant](blocks)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q4_k_hand_derived_answer():
    # d = 0.5, dmin = 0.25; scale byte 0 = 3 (sc0), byte 4 = 2 (m0); q[0] = 0x5A
    # element 0 = 0.5*3*0xA - 0.25*2 = 14.5 ; element 32 uses sub-block 1 (sc1 = 0)
    b = np.zeros(144, np.uint8)
    b[0:2] = rc.f16_bytes(0.5)
    b[2:4] = rc.f16_bytes(0.25)
    b[4] = 3
    b[8] = 2
    b[16] = 0x5A
    out = oracle.dequantize_row(Q4_K, b, 256)
    assert out[0] == np.float32(14.5)
    assert out[32] == np.float32(0.0)  # d*0*5 - dmin*0 (m1 = byte 5 & 63 = 0)
    # sub-block 4 takes its scale from the high bits: sc4 = (q[8]&15) | (q[0]>>6)<<4
    b[4] = 0xC3  # sc0 = 3, top bits 3 -> sc4 high part 3<<4 = 48
    b[12] = 0x01  # q[8] low nibble 1 -> sc4 = 49
    b[16 + 64] = 0x02  # chunk 2 (sub-block 4) element 128 -> q = 2
    out = oracle.dequantize_row(Q4_K, b, 256)
    assert out[128] == np.float32(0.5 * 49 * 2)


def test_q5_k_hand_derived_answer():
    # the qh bit 1 << (2c + hi) adds 16 (dequant.rs:290-295)
    b = np.zeros(176, np.uint8)
    b[0:2] = rc.f16_bytes(1.0)
    b[4] = 1      # sc0 = 1
    b[5] = 1      # sc1 = 1
    b[16] = 0b11  # qh[0]: bit0 -> element 0 (+16), bit1 -> element 32 (+16)
    b[48] = 0x21  # ql[0]: low 1, high 2
    out = oracle.dequantize_row(Q5_K, b, 256)
    assert out[0] == np.float32(17.0)
    assert out[32] == np.float32(18.0)


def test_f16_to_f32_all_patterns():
    L = oracle.lib()
    bits = np.arange(65536, dtype=np.uint32)
    got = np.array([L.orc_f16_to_f32(int(h)) for h in bits], np.float32)
    want = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.array_equal(np.isinf(got), np.isinf(want))
    nan = np.isnan(want)
    # NaN: payload kept, quiet bit set (half 2.7.1)
    g = got[nan].view(np.uint32)
    h = bits[nan]
    assert np.array_equal(g, ((h & 0x8000) << 16) | 0x7FC00000 | ((h & 0x3FF) << 13))


def test_bf16_round_matches_numpy_rne():
    L = oracle.lib()
    g = rng(7)
    x = np.concatenate([g.standard_normal(20000).astype(np.float32),
                        (g.integers(0, 2**32, 20000, dtype=np.uint64).astype(np.uint32) & 0x7F7FFFFF).view(np.float32)])
    # exact ties: low half = 0x8000 with even and odd high halves
    ties = (np.arange(0x3F80, 0x3F90, dtype=np.uint32) << 16 | 0x8000).view(np.float32)
    x = np.concatenate([x, ties])
    got = np.array([L.orc_f32_to_bf16_bits(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, bf16_bits(x))


def test_route_top_k_order_and_renorm():
    g = rng(3)
    logits = g.standard_normal((16, 256)).astype(np.float32)
    ids, w = oracle.route_logits(logits, 8)
    for t in range(16):
        assert np.all(np.diff(ids[t]) > 0), "ids come back in ascending order"
        lg = logits[t].astype(np.float32)
        p = np.exp((lg - lg.max()).astype(np.float32)).astype(np.float32)
        top = np.argsort(-p, kind="stable")[:8]
        assert set(top.tolist()) == set(ids[t].tolist())
        assert abs(float(w[t].astype(np.float64).sum()) - 1.0) < 1e-6


def test_route_ties_go_to_the_lower_index():
    logits = np.zeros((1, 16), np.float32)
    ids, w = oracle.route_logits(logits, 4)
    assert ids[0].tolist() == [0, 1, 2, 3]
    assert np.all(w[0] == np.float32(0.25))


def test_dequantize_row_truncation_errors():
    L = oracle.lib()
    out = np.empty(256, np.float32)
    b = np.zeros(143, np.uint8)
    assert L.orc_dequantize_row(Q4_K, b.ctypes.data, b.nbytes, oracle._fp(out), 256) == oracle.ERR_TRUNCATED
    b = np.zeros(144, np.uint8)
    assert L.orc_dequantize_row(Q4_K, b.ctypes.data, b.nbytes, oracle._fp(out), 200) == oracle.ERR_TRUNCATED
    assert L.orc_dequantize_row(99, b.ctypes.data, b.nbytes, oracle._fp(out), 256) == oracle.ERR_UNSUPPORTED


def test_threaded_gemv_equals_single_thread():
    w = quant_blocks(rng(11), Q4_K, 64 * 8).reshape(-1)
    x = rng(12).standard_normal((2, 2048)).astype(np.float32)
    a = oracle.gemv(Q4_K, w, 64, 2048, x, threads=1)
    b = oracle.gemv(Q4_K, w, 64, 2048, x, threads=4)
    assert np.array_equal(a, b)


# ---- the elementwise trait methods: the reference's own known values
# (crates/strata-core/tests/ops_tests.rs:80-134) and a numpy f64 restatement

def test_rms_norm_known_values():
    """ops_tests.rs:80-88: [3, 4] with w = [2, 2], eps 0 -> [3, 4] * 2 / sqrt(12.5)."""
    got = oracle.rms_norm(np.array([3.0, 4.0], np.float32), np.array([2.0, 2.0], np.float32), 0.0)
    s = 2.0 / np.sqrt(12.5)
    assert abs(got[0] - np.float32(3.0 * s)) < 1e-6 and abs(got[1] - np.float32(4.0 * s)) < 1e-6


def test_l2_norm_gives_unit_heads():
    """ops_tests.rs:90-96."""
    got = oracle.l2_norm(np.array([3.0, 4.0, 0.0], np.float32), 3, 0.0)
    assert abs(float(np.sqrt(np.sum(got * got))) - 1.0) < 1e-6


def test_rope_neox_known_values():
    """ops_tests.rs:98-125: position 0 is the identity; (1, 0) at pos 1, base 1 -> (cos 1, sin 1)."""
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    assert np.array_equal(oracle.rope_neox(x, 4, 0, 4, 1e7), x)
    got = oracle.rope_neox(np.array([1.0, 0.0], np.float32), 2, 1, 2, 1.0)
    assert abs(got[0] - np.float32(np.cos(1.0))) < 1e-6 and abs(got[1] - np.float32(np.sin(1.0))) < 1e-6


def test_softmax_sums_to_one():
    """ops_tests.rs:127-134."""
    got = oracle.softmax(np.array([1.0, 2.0, 3.0, 0.5], np.float32), 4)
    assert abs(float(np.sum(got.astype(np.float64))) - 1.0) < 1e-6
    assert got[2] > got[1] > got[0] > got[3]


def test_silu_and_sigmoid_known_values():
    """ops_tests.rs:137-143 (silu and sigmoid; softplus is not on this path)."""
    assert abs(oracle.lib().orc_silu(0.0)) < 1e-7
    assert abs(oracle.lib().orc_sigmoid(0.0) - 0.5) < 1e-7


def test_q2_0_structural_invariant():
    """Every Q2_0 output is one of -d, 0, +d, +2d."""
    out = oracle.dequantize_row(synth.Q2_0, rc.q2_0_invariant_block(), 64)
    d = 0.5
    assert all(min(abs(v + d), abs(v), abs(v - d), abs(v - 2 * d)) < 1e-6 for v in out)


def test_elementwise_ops_match_numpy_f64():
    """The same arithmetic restated in numpy (f64 where ops.rs uses f64)."""
    g = rng(77)
    x = g.standard_normal((3, 256)).astype(np.float32)
    w = g.standard_normal(256).astype(np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=1, keepdims=True) / 256
    want = ((x.astype(np.float64) * (1.0 / np.sqrt(ss + 1e-6))) * w.astype(np.float64)).astype(np.float32)
    assert np.max(np.abs(oracle.rms_norm(x, w, 1e-6) - want)) <= 1e-6 * np.max(np.abs(want))
    h = x.reshape(-1, 128)
    inv = 1.0 / np.sqrt(np.sum(h.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)
    assert np.max(np.abs(oracle.l2_norm(h, 128, 1e-6) - (h * inv).astype(np.float32))) < 1e-6
    e = np.exp((x - x.max(axis=1, keepdims=True)).astype(np.float64))
    assert np.max(np.abs(oracle.softmax(x, 256) - (e / e.sum(axis=1, keepdims=True)).astype(np.float32))) < 1e-6
    half = 32
    th = 1e6 ** (-2.0 * np.arange(half) / 64) * 17
    a, b = h[:, :half].astype(np.float64), h[:, half:2 * half].astype(np.float64)
    r = oracle.rope_neox(h, 128, 17, 64, 1e6)
    assert np.max(np.abs(r[:, :half] - (a * np.cos(th) - b * np.sin(th)))) < 1e-5
    assert np.max(np.abs(r[:, half:2 * half] - (a * np.sin(th) + b * np.cos(th)))) < 1e-5
    assert np.array_equal(r[:, 64:], h[:, 64:])
    assert np.array_equal(oracle.add(x, w[None, :].repeat(3, 0)), x + w)


@pytest.mark.parametrize("quant", synth.OTHER_FORMATS)
def test_other_formats_match_independent_numpy_restatement(quant):
    """The formats beyond the benchmark's four, oracle vs the numpy restatement, bit for bit."""
    g = rng(600 + quant)
    blocks = synth.quant_blocks(g, quant, 256)
    bs, _ = synth.BLOCK[quant]
    got = oracle.dequantize_row(quant, blocks.reshape(-1), blocks.shape[0] * bs)
    want = numpy_dequant.DEQUANT[quant](blocks)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("bad", [np.nan, np.inf])
def test_route_with_a_nan_or_inf_logit_falls_back_to_index_order(bad):
    """MoeLayer::route (moe.rs:57-91) on a NaN or +Inf logit: the max-shifted
    exp of that logit is NaN (inf - inf), so the f64 sum, the f32 reciprocal and
    every probability are NaN; the comparator's partial_cmp then yields Equal
    for every pair and the index decides: ids 0..k-1. Their weights are NaN
    (NaN / max(NaN, 2^-14) = NaN / 2^-14). A -Inf logit is an ordinary zero."""
    E, k = 64, 8
    lg = rng(91).standard_normal((3, E)).astype(np.float32)
    lg[0, 17] = bad
    lg[1, :] = bad
    lg[2, 5] = -np.inf
    ids, w = oracle.route_logits(lg, k)
    for t in (0, 1):
        assert np.array_equal(ids[t], np.arange(k))
        assert np.all(np.isnan(w[t]))
    assert 5 not in ids[2]
    p = np.exp((lg[2] - lg[2].max()).astype(np.float64))
    want = np.sort(np.argsort(-p, kind="stable")[:k])
    assert np.array_equal(ids[2], want)


def test_expf_helpers_find_where_the_c_library_is_not_correctly_rounded():
    """The reference's f32::exp is the C library's expf, which misrounds a few
    inputs (its error bound is 0.502 ulp). The test-support scans return
    inputs where expf differs from the correctly rounded exp (the double exp
    rounded to f32: the two agree on every float of [-104, 0]), and pairs a few
    floats apart that expf ties and the correctly rounded exp separates."""
    import ctypes
    import math
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype, libm.expf.argtypes = ctypes.c_float, [ctypes.c_float]

    def expf(v):
        return np.float32(libm.expf(float(v)))

    m = oracle.expf_misrounded(-1.0, -0.5, 10**6)
    assert 100 < m.size < 10**5
    for v in m[:: max(1, m.size // 200)]:
        assert expf(v) != np.float32(math.exp(float(v))), v
    pairs = oracle.expf_tie_pairs(-1.0, -0.5, 32)
    assert len(pairs) == 32
    for a, b in pairs:
        assert a < b and expf(a) == expf(b)
        assert np.float32(math.exp(float(a))) < np.float32(math.exp(float(b)))
