"""Parity of the device MoE layer (through the C ABI) with the CPU oracle.

MoeLayer::route + MoeLayer::combine (crates/strata-core/src/moe.rs:48-144):
routing from given logits is compared exactly (ids) and to the bit or one
ulp (weights); the layer output within rel_err 1e-3 (fp32 accumulation
against the reference's f32/f64 mix).
"""
import math

import numpy as np
import pytest

import oracle
import strata_cuda as sc
from conftest import rel_err
from synth import Q4_K, Q5_K, Q6_K, Q8_0, F32, activations, bf16_round, quant_matrix, rng

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = sc.Context(0)
    yield c
    c.close()


def make_layer(seed, n_embd, E, n_ff, n_ff_s, qe=Q4_K, qs=Q4_K, qr=Q4_K, shared=True, router=True):
    t = {}
    if router:
        t["router"] = (qr, quant_matrix(seed, qr, E, n_embd))
    t["gate_exps"] = (qe, quant_matrix(seed + 1, qe, n_embd, n_ff, E))
    t["up_exps"] = (qe, quant_matrix(seed + 2, qe, n_embd, n_ff, E))
    t["down_exps"] = (qe, quant_matrix(seed + 3, qe, n_ff, n_embd, E))
    if shared:
        t["gate_shexp"] = (qs, quant_matrix(seed + 4, qs, n_ff_s, n_embd))
        t["up_shexp"] = (qs, quant_matrix(seed + 5, qs, n_ff_s, n_embd))
        t["down_shexp"] = (qs, quant_matrix(seed + 6, qs, n_embd, n_ff_s))
        t["gate_inp_shexp"] = (qs, quant_matrix(seed + 7, qs, 1, n_embd))
    return t


SHAPE = {"router": lambda d: (d["E"], d["n_embd"], 0), "gate_exps": lambda d: (d["n_embd"], d["n_ff"], d["E"]),
         "up_exps": lambda d: (d["n_embd"], d["n_ff"], d["E"]), "down_exps": lambda d: (d["n_ff"], d["n_embd"], d["E"]),
         "gate_shexp": lambda d: (d["n_ff_s"], d["n_embd"], 0), "up_shexp": lambda d: (d["n_ff_s"], d["n_embd"], 0),
         "down_shexp": lambda d: (d["n_embd"], d["n_ff_s"], 0), "gate_inp_shexp": lambda d: (1, d["n_embd"], 0)}


def upload(ctx, t, dims, e0=0, e1=None):
    """Uploads the tensors; expert tensors restricted to experts [e0, e1)."""
    ws = {}
    for nm, (q, arr) in t.items():
        rows, cols, ne = SHAPE[nm](dims)
        if ne:
            e1_ = ne if e1 is None else e1
            per = arr.size // ne
            ws[nm] = ctx.upload(arr[e0 * per:e1_ * per], q, rows, cols, n_expert=e1_ - e0)
        else:
            ws[nm] = ctx.upload(arr, q, rows, cols)
    return ws


def free_all(ws, layer=None):
    if layer is not None:
        layer.free()
    for w in ws.values():
        w.free()


def check_routing(ids, wts, want_ids, want_w):
    assert np.array_equal(ids.astype(np.int64), want_ids)
    # weights: the same f32 operations; exp may differ from the host's expf by an ulp
    d = np.abs(wts.view(np.int32).astype(np.int64) - want_w.view(np.int32).astype(np.int64))
    assert d.max() <= 2, d.max()


@pytest.mark.parametrize("T", [1, 2, 3, 17])
@pytest.mark.parametrize("qe", [Q4_K, Q5_K, Q6_K, Q8_0])
def test_moe_small_from_logits(ctx, T, qe, threads):
    dims = dict(n_embd=512, E=16, k=4, n_ff=256, n_ff_s=256)
    t = make_layer(1000 + qe, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"], qe=qe)
    ws = upload(ctx, t, dims)
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    x = activations(1001 + T, T, dims["n_embd"])
    logits = rng(1002 + T).standard_normal((T, dims["E"])).astype(np.float32)
    out, ids, w = ctx.moe_ffn(layer, x, logits)
    want, want_ids, want_w = oracle.moe_layer(t, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                                              x, logits, threads=threads)
    check_routing(ids, w, want_ids, want_w)
    for i in range(T):
        assert rel_err(out[i], want[i]) < TOL, (i, rel_err(out[i], want[i]))
    free_all(ws, layer)


def test_moe_routing_with_nan_and_inf_logits(ctx, threads):
    """A NaN or +Inf router logit makes every probability NaN (the f64 sum is
    NaN): the reference then picks experts 0..k-1 in index order with NaN
    weights. The device must pick the same ids and stay inside the expert
    array; tokens with ordinary logits route as usual."""
    dims = dict(n_embd=512, E=64, k=8, n_ff=256, n_ff_s=256)
    t = make_layer(1500, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"])
    ws = upload(ctx, t, dims)
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    T = 4
    x = activations(1501, T, dims["n_embd"])
    logits = rng(1502).standard_normal((T, dims["E"])).astype(np.float32)
    logits[0, 33] = np.nan
    logits[1, 2] = np.inf
    logits[2, :] = np.nan
    logits[3, 7] = -np.inf
    out, ids, w = ctx.moe_ffn(layer, x, logits)
    want, want_ids, want_w = oracle.moe_layer(t, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                                              x, logits, threads=threads)
    assert np.array_equal(ids.astype(np.int64), want_ids)
    for tok in (0, 1, 2):
        assert np.array_equal(want_ids[tok], np.arange(dims["k"]))
        assert np.all(np.isnan(w[tok])) and np.all(np.isnan(want_w[tok]))
        assert np.array_equal(np.isnan(out[tok]), np.isnan(want[tok]))
    check_routing(ids[3:], w[3:], want_ids[3:], want_w[3:])
    assert rel_err(out[3], want[3]) < TOL
    free_all(ws, layer)


def test_moe_routing_exp_is_the_c_librarys_expf(ctx, threads):
    """The router's f32::exp is the C library's expf, not the correctly
    rounded exp (they differ on about 1 in 11,500 inputs of the max-shifted
    domain). (a) Logit rows of one 0 and 63 inputs where expf is misrounded,
    all in [-8, 0] so the f64 sums are exact in any order: ids and weights are
    the oracle's bits. (b) The top-k boundary: experts 3 and 9 get two logits
    a few floats apart on which expf ties but the correctly rounded exp does
    not; the reference's tie goes to the lower index (expert 3), a correctly
    rounded exp would take expert 9. The device must take expert 3."""
    dims = dict(n_embd=512, E=64, k=8, n_ff=256, n_ff_s=256)
    t = make_layer(1600, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"])
    ws = upload(ctx, t, dims)
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    T = 16
    m = oracle.expf_misrounded(-8.0, -0.25, T * 63)
    assert m.size == T * 63
    logits = np.zeros((T, dims["E"]), np.float32)
    logits[:, 1:] = rng(1601).permutation(m).reshape(T, 63)
    x = activations(1602, T, dims["n_embd"])
    _, ids, w = ctx.moe_ffn(layer, x, logits)
    want_ids, want_w = oracle.route_logits(logits, dims["k"])
    assert np.array_equal(ids.astype(np.int64), want_ids)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))

    pairs = oracle.expf_tie_pairs(-2.0, -0.25, T)
    assert len(pairs) == T
    k = 4
    logits = np.full((T, dims["E"]), -3.0, np.float32)
    logits[:, 0], logits[:, 1], logits[:, 2] = 0.0, -0.01, -0.02   # the first three picks
    logits[:, 3], logits[:, 9] = pairs[:, 0], pairs[:, 1]           # x1 < x2: expf(x1) == expf(x2)
    layer4 = ctx.moe_create(ws, dims["n_embd"], dims["E"], k, dims["n_ff"], dims["n_ff_s"])
    _, ids, w = ctx.moe_ffn(layer4, x, logits)
    want_ids, want_w = oracle.route_logits(logits, k)
    assert np.array_equal(want_ids, np.tile([0, 1, 2, 3], (T, 1)))  # the tie to the lower index
    # a correctly rounded exp separates the pair: expert 9 would come fourth
    cr = np.float32([[math.exp(float(v)) for v in row] for row in logits])
    assert np.all(cr[:, 9] > cr[:, 3])
    assert np.array_equal(ids.astype(np.int64), want_ids)
    assert np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    layer4.free()
    free_all(ws, layer)


def test_moe_router_gemv_path(ctx, threads):
    dims = dict(n_embd=512, E=32, k=4, n_ff=256, n_ff_s=256)
    t = make_layer(1100, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"])
    ws = upload(ctx, t, dims)
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    T = 9
    x = activations(1101, T, dims["n_embd"])
    out, ids, w = ctx.moe_ffn(layer, x, None)
    want, want_ids, want_w = oracle.moe_layer(t, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                                              x, None, threads=threads)
    # the router GEMV accumulates in f32 (the reference in f64): routing may only
    # differ where the k-th and (k+1)-th probabilities are within that noise
    lg = oracle.gemv(Q4_K, t["router"][1], dims["E"], dims["n_embd"], bf16_round(x), threads=threads)
    for i in range(T):
        srt = np.sort(lg[i])[::-1]
        if srt[dims["k"] - 1] - srt[dims["k"]] < 1e-4 * max(1.0, abs(srt[0])):
            continue
        assert np.array_equal(ids[i], want_ids[i])
        # weights go as exp(logit): the logits' f32 noise (~1e-6 of their
        # magnitude, here tens) moves them by ~1e-5 relative, and the output
        # inherits that through w * down (outputs here reach ~7e4, the
        # metric's floor is 1e-3 of that): the kernels' own 1e-3 parity is
        # checked on given logits above
        assert np.allclose(w[i], want_w[i], rtol=1e-3, atol=0)
        assert rel_err(out[i], want[i]) < 1e-2
    free_all(ws, layer)


@pytest.mark.parametrize("T", [1, 64])
def test_moe_config_layer(ctx, T, threads):
    """The MoE FFN configuration: hidden 2048, 256 experts of SwiGLU width 512,
    top-8 from N(0,1) logits, a shared expert of width 512, all Q4_K."""
    dims = dict(n_embd=2048, E=256, k=8, n_ff=512, n_ff_s=512)
    t = make_layer(1200, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"], router=False)
    ws = upload(ctx, t, dims)
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    x = activations(1201 + T, T, dims["n_embd"])
    logits = rng(1202 + T).standard_normal((T, dims["E"])).astype(np.float32)
    out, ids, w = ctx.moe_ffn(layer, x, logits)
    want, want_ids, want_w = oracle.moe_layer(t, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                                              x, logits, threads=threads)
    check_routing(ids, w, want_ids, want_w)
    errs = [rel_err(out[i], want[i]) for i in range(T)]
    assert max(errs) < TOL, max(errs)
    # deterministic run to run
    out2, _, _ = ctx.moe_ffn(layer, x, logits)
    assert np.array_equal(out.view(np.uint32), out2.view(np.uint32))
    free_all(ws, layer)


@pytest.mark.parametrize("G", [2, 4])
def test_moe_expert_parallel_partials_sum(ctx, G):
    """Expert parallelism on one GPU: G layers over expert slices (the shared
    expert in the first) produce partial outputs whose sum is the layer."""
    dims = dict(n_embd=512, E=32, k=4, n_ff=256, n_ff_s=256)
    t = make_layer(1300, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"], router=False)
    T = 11
    x = activations(1301, T, dims["n_embd"])
    logits = rng(1302).standard_normal((T, dims["E"])).astype(np.float32)
    ws = upload(ctx, t, dims)
    full = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    want, want_ids, want_w = ctx.moe_ffn(full, x, logits)
    total = np.zeros_like(want)
    per = dims["E"] // G
    for r in range(G):
        wr = upload(ctx, {k: v for k, v in t.items()}, dims, e0=r * per, e1=(r + 1) * per)
        lr = ctx.moe_create(wr, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                            expert_begin=r * per, expert_end=(r + 1) * per, with_shared=(r == 0))
        part, ids, w = ctx.moe_ffn(lr, x, logits)
        assert np.array_equal(ids, want_ids) and np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
        total += part
        free_all(wr, lr)
    # both are fp32 sums, in different orders (the row split depends on the experts
    # held); outputs here reach ~3e4, so the near-zero floor (1e-3 |ref|inf) sees
    # their rounding: compare at the parity bar
    for i in range(T):
        assert rel_err(total[i], want[i]) < TOL
    free_all(ws, full)


@pytest.mark.parametrize("q", [Q4_K, Q5_K])
@pytest.mark.parametrize("G", [1, 2, 4])
def test_moe_one_token_layer(ctx, q, G, threads):
    """One token (the decode chain: routing with assignment, the few-token
    gate/up and down passes, the combine) with every expert and shared tensor
    Q4_K or every one Q5_K, 64 experts, top-8: the output against the oracle's
    layer and, over expert slices (G > 1, the shared expert in the first), the
    partial outputs summing to it; routing identical on every slice, on two
    calls in a row."""
    dims = dict(n_embd=1024, E=64, k=8, n_ff=512, n_ff_s=256)
    t = make_layer(1700 + q, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"], qe=q, qs=q, router=False)
    x = activations(1701, 1, dims["n_embd"])
    logits = rng(1702 + G).standard_normal((1, dims["E"])).astype(np.float32)
    want, want_ids, want_w = oracle.moe_layer(t, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                                              x, logits, threads=threads)
    total = np.zeros_like(want)
    per = dims["E"] // G
    for r in range(G):
        ws = upload(ctx, t, dims, e0=r * per, e1=(r + 1) * per)
        layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"],
                               expert_begin=r * per, expert_end=(r + 1) * per, with_shared=(r == 0))
        for call in range(2):
            part, ids, w = ctx.moe_ffn(layer, x, logits)
            check_routing(ids, w, want_ids, want_w)
        total += part
        free_all(ws, layer)
    assert rel_err(total[0], want[0]) < TOL, rel_err(total[0], want[0])


def test_moe_host_calls_replay_captured_graphs(threads):
    """The host-buffer layer call captures its work (input copy, both streams'
    launches, output copy) as a graph per token count and replays it on later
    calls with that count. Over more token counts than the cache keeps, with
    and without router logits, a replayed call on new inputs matches the
    oracle, and a replayed call on the first inputs equals the direct first
    call bit for bit. A context destroyed before its layer releases the
    layer's graphs (the layer is freed afterwards)."""
    dims = dict(n_embd=512, E=16, k=4, n_ff=256, n_ff_s=256)
    t = make_layer(1600, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"])
    c = sc.Context(0)
    ws = upload(c, t, dims)
    layer = c.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    checked = 0
    for n, T in enumerate([1, 2, 3, 5, 7, 1, 3]):
        for with_logits in (True, False):
            xa = activations(1601 + n, T, dims["n_embd"])
            xb = activations(1651 + n, T, dims["n_embd"])
            la = rng(1701 + n).standard_normal((T, dims["E"])).astype(np.float32) if with_logits else None
            lb = rng(1751 + n).standard_normal((T, dims["E"])).astype(np.float32) if with_logits else None
            first = c.moe_ffn(layer, xa, la)
            other = c.moe_ffn(layer, xb, lb)
            again = c.moe_ffn(layer, xa, la)
            for u, v in zip(first, again):
                assert np.array_equal(u.view(np.uint32), v.view(np.uint32)), (T, with_logits)
            if with_logits and checked < 3:
                want, want_ids, want_w = oracle.moe_layer(t, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"],
                                                          dims["n_ff_s"], xb, lb, threads=threads)
                check_routing(other[1], other[2], want_ids, want_w)
                for i in range(T):
                    assert rel_err(other[0][i], want[i]) < TOL, (T, i)
                checked += 1
    # a change of GEMV path reaches the router and shared-expert GEMVs of a
    # token count already cached: the host call then equals the (never
    # cached) device-buffer call on the new path
    torch = pytest.importorskip("torch")
    x = activations(1850, 2, dims["n_embd"])
    c.moe_ffn(layer, x)
    c.moe_ffn(layer, x)
    c.set_gemv_path(sc.Context.GEMV_CUDA_CORES)
    host = c.moe_ffn(layer, x)[0]
    xd = torch.from_numpy(x).cuda()
    od = torch.empty((2, dims["n_embd"]), dtype=torch.float32, device="cuda")
    c.moe_ffn_dev(layer, xd.data_ptr(), 0, 2, od.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(host.view(np.uint32), od.cpu().numpy().view(np.uint32))
    c.set_gemv_path(sc.Context.GEMV_AUTO)
    c2 = sc.Context(0)
    ws2 = upload(c2, t, dims)
    layer2 = c2.moe_create(ws2, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    x = activations(1800, 2, dims["n_embd"])
    r1 = c2.moe_ffn(layer2, x)
    r2 = c2.moe_ffn(layer2, x)
    assert np.array_equal(r1[0].view(np.uint32), r2[0].view(np.uint32))
    c2.close()
    layer2.free()
    free_all(ws, layer)
    c.close()


def test_moe_dev_entry_on_torch_stream(ctx):
    torch = pytest.importorskip("torch")
    dims = dict(n_embd=512, E=16, k=4, n_ff=256, n_ff_s=256)
    t = make_layer(1400, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"], router=False)
    ws = upload(ctx, t, dims)
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    T = 5
    x = activations(1401, T, dims["n_embd"])
    logits = rng(1402).standard_normal((T, dims["E"])).astype(np.float32)
    host, _, _ = ctx.moe_ffn(layer, x, logits)
    xd, ld = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
    od = torch.empty((T, dims["n_embd"]), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ctx.moe_ffn_dev(layer, xd.data_ptr(), ld.data_ptr(), T, od.data_ptr(), stream=s.cuda_stream)
    s.synchronize()
    assert np.array_equal(od.cpu().numpy().view(np.uint32), host.view(np.uint32))
    free_all(ws, layer)


def test_moe_rejects(ctx):
    dims = dict(n_embd=512, E=16, k=4, n_ff=256, n_ff_s=256)
    t = make_layer(1500, dims["n_embd"], dims["E"], dims["n_ff"], dims["n_ff_s"], router=False)
    ws = upload(ctx, t, dims)
    with pytest.raises(sc.BackendError) as e:
        ctx.moe_create(ws, dims["n_embd"], dims["E"], 33, dims["n_ff"], dims["n_ff_s"])
    assert e.value.code == sc.ERR_INVALID
    with pytest.raises(sc.BackendError) as e:  # down_exps passed as gate_exps: wrong shape
        ctx.moe_create(dict(ws, gate_exps=ws["down_exps"]), dims["n_embd"], dims["E"], 4, dims["n_ff"], dims["n_ff_s"])
    assert e.value.code == sc.ERR_INVALID
    layer = ctx.moe_create(ws, dims["n_embd"], dims["E"], dims["k"], dims["n_ff"], dims["n_ff_s"])
    with pytest.raises(sc.BackendError) as e:  # no router weight and no logits
        ctx.moe_ffn(layer, activations(1, 2, dims["n_embd"]), None)
    assert e.value.code == sc.ERR_INVALID
    free_all(ws, layer)
    fe = ctx.upload(np.zeros(16 * 512 * 256 * 4, np.uint8), F32, 512, 256, n_expert=16)
    with pytest.raises(sc.BackendError) as e:
        ctx.moe_create(dict(gate_exps=fe, up_exps=fe, down_exps=fe), 512, 16, 4, 256)
    assert e.value.code in (sc.ERR_UNSUPPORTED_QUANT, sc.ERR_INVALID)
    fe.free()
