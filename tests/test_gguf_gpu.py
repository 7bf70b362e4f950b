"""GGUF ingest to HBM: a model split over two shards is opened by the reader
and its tensors are uploaded in one staged pass (strata_cuda_gguf_ingest over
strata_cuda_upload_many), viewed as strata-core's WeightStore views them
(crates/strata-core/src/weights.rs:122-152). Every tensor must arrive byte for
byte: its dequantized rows, for every expert, equal the oracle's dequant of
the file's bytes bit for bit, and a GEMV on an ingested matrix meets the
1e-3 tolerance. Batched uploads are all or nothing."""
import time

import numpy as np
import pytest

import oracle
import strata_cuda as sc
from conftest import rel_err
from gguf_writer import STRING, U32, build
from synth import activations, quant_blocks, quant_matrix, rng

pytestmark = pytest.mark.gpu
IQ2_XXS = 16  # read by the GGUF reader, not on the device path

SHARD1 = [("blk.0.attn_q.weight", [2048, 512], sc.Q4_K), ("blk.0.attn_k.weight", [4096, 96], sc.Q8_0),
          ("blk.0.ffn_down.weight", [512, 300], sc.Q6_K), ("blk.0.attn_norm.weight", [2048], sc.F32),
          ("blk.0.attn_v.weight", [256, 4], IQ2_XXS)]
SHARD2 = [("blk.0.ffn_gate_exps.weight", [512, 2048, 128], sc.Q4_K),
          ("blk.0.ffn_down_exps.weight", [2048, 512, 8], sc.Q5_K),
          ("blk.0.ffn_up_exps.weight", [512, 2048, 3], sc.Q6_K), ("output_norm.weight", [512], sc.Q8_0)]


def payload(g, quant, shape):
    n = int(np.prod(shape))
    if quant == sc.F32:
        return g.standard_normal(n).astype(np.float32).tobytes()
    if quant == IQ2_XXS:
        return g.integers(0, 256, n // 256 * 66, dtype=np.uint8).tobytes()
    return quant_blocks(g, quant, n // sc.BLOCK[quant][0]).reshape(-1).tobytes()


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    d = tmp_path_factory.mktemp("gguf")
    g = rng(2718)
    blobs = {}
    for k, (spec, meta) in enumerate([(SHARD1, [("general.architecture", STRING, "qwen35moe"),
                                                ("split.count", U32, 2), ("split.no", U32, 0)]),
                                      (SHARD2, [("split.count", U32, 2), ("split.no", U32, 1)])]):
        tensors = []
        for name, shape, quant in spec:
            blobs[name] = payload(g, quant, shape)
            tensors.append((name, shape, quant, blobs[name]))
        data, _, _ = build(meta, tensors)
        (d / f"synth-{k + 1:05d}-of-00002.gguf").write_bytes(data)
    m = sc.GgufModel(d / "synth-00002-of-00002.gguf")
    yield m, blobs
    m.close()


@pytest.fixture(scope="module")
def ctx():
    c = sc.Context(0)
    yield c
    c.close()


def test_ingest_round_trips_every_tensor(ctx, model):
    m, blobs = model
    names = [n for n, _, q in SHARD1 + SHARD2 if q != IQ2_XXS]
    total = sum(len(blobs[n]) for n in names)
    before = ctx.resident_bytes()
    for w in ctx.ingest(m, names).values():  # the first staged upload pins the staging chunks
        w.free()
    t0 = time.perf_counter()
    ws = ctx.ingest(m, names)
    dt = time.perf_counter() - t0
    print(f"ingest {len(names)} tensors, {total / 1e6:.0f} MB from 2 shards in {dt * 1e3:.1f} ms: "
          f"{total / dt / 1e9:.1f} GB/s")
    assert ctx.resident_bytes() - before == total
    for name in names:
        t, w = m.find(name), ws[name]
        data = np.frombuffer(blobs[name], np.uint8)
        assert np.array_equal(m.tensor_data(name), data)
        rb = sc.byte_size(t.ty, w.cols)
        for e in range(max(1, w.n_expert)):
            got = ctx.dequant(w, expert=e)
            part = data[e * w.rows * rb:(e + 1) * w.rows * rb]
            want = oracle.dequantize(t.ty, part, w.rows, w.cols)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (name, e)
    q = ws["blk.0.attn_q.weight"]
    x = activations(31, 2, q.cols)
    y = ctx.gemv(q, x)
    want = oracle.gemv(sc.Q4_K, np.frombuffer(blobs["blk.0.attn_q.weight"], np.uint8), q.rows, q.cols, x, threads=4)
    for b in range(2):
        assert rel_err(y[b], want.reshape(2, q.rows)[b]) < 1e-3
    for w in ws.values():
        w.free()
    assert ctx.resident_bytes() == before


def test_ingest_is_all_or_nothing(ctx, model):
    m, _ = model
    before = ctx.resident_bytes()
    with pytest.raises(sc.BackendError) as ei:
        ctx.ingest(m, ["blk.0.attn_q.weight", "blk.0.attn_v.weight"])
    assert ei.value.code == sc.ERR_UNSUPPORTED_QUANT and "blk.0.attn_v.weight" in str(ei.value)
    assert ctx.resident_bytes() == before


def test_upload_many_small_ranges_across_chunks(ctx):
    """70 Q8_0 matrices of odd sizes, 100+ MB in all: chunk boundaries fall
    inside tensors and several tensors share a chunk."""
    g = rng(99)
    cols = 1024
    rb = cols // 32 * 34
    items, datas = [], []
    for k in range(70):
        rows = int(g.integers(1, 3000))
        d = quant_blocks(g, sc.Q8_0, rows * cols // 32).reshape(-1)
        datas.append(d)
        items.append((d, sc.Q8_0, rows, cols, 0))
    assert sum(d.nbytes for d in datas) > 96 << 20
    before = ctx.resident_bytes()
    ws = ctx.upload_many(items)
    for d, (_, _, rows, _, _), w in zip(datas, items, ws):
        got = ctx.dequant(w)
        want = oracle.dequantize(sc.Q8_0, d, rows, cols)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert rb * rows == d.nbytes
    for w in ws:
        w.free()
    # an invalid item (cols not whole blocks) refuses the whole batch
    bad = items[:5] + [(datas[5], sc.Q8_0, items[5][2], cols - 1, 0)] + items[6:9]
    with pytest.raises(sc.BackendError) as ei:
        ctx.upload_many(bad)
    assert ei.value.code == sc.ERR_TRUNCATED and "upload 5 of 9" in str(ei.value)
    assert ctx.resident_bytes() == before


def test_rank_slices_upload_only_their_bytes(ctx, model):
    """A rank of a row-sharded projection or of the expert-parallel MoE uploads
    its own slice straight from the mapping (strata_cuda_gguf_view +
    strata_cuda_upload_many); the slice dequantizes as the matching rows or
    experts of the whole tensor."""
    import sharding
    m, blobs = model
    world, rank = 4, 1
    before = ctx.resident_bytes()
    views = [sharding.row_shard_view(m, "blk.0.attn_q.weight", world, rank),
             sharding.expert_shard_view(m, "blk.0.ffn_gate_exps.weight", world, rank)]
    dense, exps = ctx.upload_views(views)
    assert ctx.resident_bytes() - before == views[0].len + views[1].len
    q = np.frombuffer(blobs["blk.0.attn_q.weight"], np.uint8)
    rb = sc.byte_size(sc.Q4_K, 2048)
    r0, r1 = sharding.row_range(512, world, rank)
    want = oracle.dequantize(sc.Q4_K, q[r0 * rb:r1 * rb], r1 - r0, 2048)
    assert np.array_equal(ctx.dequant(dense).view(np.uint32), want.view(np.uint32))
    ge = np.frombuffer(blobs["blk.0.ffn_gate_exps.weight"], np.uint8)
    e0, e1 = sharding.expert_range(128, world, rank)
    per = 2048 * sc.byte_size(sc.Q4_K, 512)
    for k in (0, e1 - e0 - 1):
        got = ctx.dequant(exps, expert=k)
        want = oracle.dequantize(sc.Q4_K, ge[(e0 + k) * per:(e0 + k + 1) * per], 2048, 512)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), k
    dense.free()
    exps.free()
    assert ctx.resident_bytes() == before


def test_moe_layer_from_a_gguf_file(ctx, tmp_path):
    """strata_cuda_gguf_moe_layer: a layer's tensors found by name in a GGUF
    file (load_layer, crates/strata-core/src/moe.rs:147-188), uploaded in one
    pass, run on the device against the oracle's layer on the same bytes."""
    n_embd, E, k, n_ff, n_ffs = 256, 8, 2, 256, 256
    t = {"router": (sc.Q4_K, quant_matrix(7001, sc.Q4_K, E, n_embd)),
         "gate_exps": (sc.Q4_K, quant_matrix(7002, sc.Q4_K, n_embd, n_ff, E)),
         "up_exps": (sc.Q4_K, quant_matrix(7003, sc.Q4_K, n_embd, n_ff, E)),
         "down_exps": (sc.Q4_K, quant_matrix(7004, sc.Q4_K, n_ff, n_embd, E)),
         "gate_shexp": (sc.Q4_K, quant_matrix(7005, sc.Q4_K, n_ffs, n_embd)),
         "up_shexp": (sc.Q4_K, quant_matrix(7006, sc.Q4_K, n_ffs, n_embd)),
         "down_shexp": (sc.Q4_K, quant_matrix(7007, sc.Q4_K, n_embd, n_ffs)),
         "gate_inp_shexp": (sc.Q4_K, quant_matrix(7008, sc.Q4_K, 1, n_embd))}
    gguf = {"router": ("ffn_gate_inp", [n_embd, E]), "gate_exps": ("ffn_gate_exps", [n_ff, n_embd, E]),
            "up_exps": ("ffn_up_exps", [n_ff, n_embd, E]), "down_exps": ("ffn_down_exps", [n_embd, n_ff, E]),
            "gate_shexp": ("ffn_gate_shexp", [n_embd, n_ffs]), "up_shexp": ("ffn_up_shexp", [n_embd, n_ffs]),
            "down_shexp": ("ffn_down_shexp", [n_ffs, n_embd]), "gate_inp_shexp": ("ffn_gate_inp_shexp", [n_embd])}
    tensors = [(f"blk.0.{gguf[nm][0]}.weight", gguf[nm][1], q, arr.tobytes()) for nm, (q, arr) in t.items()]
    data, _, _ = build([("general.architecture", STRING, "qwen35moe")], tensors)
    (tmp_path / "layer.gguf").write_bytes(data)
    before = ctx.resident_bytes()
    with sc.GgufModel(tmp_path / "layer.gguf") as m:
        layer, ws = ctx.gguf_moe_layer(m, 0, k)
    assert len(ws) == 8
    x = activations(7009, 3, n_embd)
    logits = rng(7010).standard_normal((3, E)).astype(np.float32)
    out, ids, w = ctx.moe_ffn(layer, x, logits)
    want, want_ids, _ = oracle.moe_layer(t, n_embd, E, k, n_ff, n_ffs, x, logits)
    assert np.array_equal(ids, want_ids.astype(np.int32))
    for i in range(3):
        assert rel_err(out[i], want[i]) < 1e-3, i
    layer.free()
    for wt in ws:
        wt.free()
    assert ctx.resident_bytes() == before
