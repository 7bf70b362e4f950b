"""The GGUF reader of the ingest path (include/strata_gguf.h) on the CPU.

It restates strata-gguf's reader (crates/strata-gguf/src/reader.rs), so these
tests restate the reference's own reader tests (crates/strata-gguf/tests/
reader_tests.rs:201-333: read-back, bad magic, split-path resolution, a model
split over two shards) and then walk every check the reference makes, each
with the error it raises (crates/strata-gguf/src/error.rs): truncation at every
byte, version, key length, UTF-8, value types, nesting, array limits,
duplicate and malformed tensors, alignment, metadata-only shards and the
payload bounds. Files are written by tests/gguf_writer.py. No GPU is used.
"""
import struct

import numpy as np
import pytest

import oracle
import strata_cuda as sc
from gguf_writer import (ARRAY, BOOL, F32, F64, I8, I16, I32, I64, STRING, U8, U16, U32, U64, build, gstring, kv,
                         q8_0_block, tensor_info)
from synth import rng

Q8_0, Q4_K, F32_T = sc.Q8_0, sc.Q4_K, sc.F32


def write(tmp_path, name, data: bytes):
    p = tmp_path / name
    p.write_bytes(data)
    return p


def open_err(path) -> sc.BackendError:
    with pytest.raises(sc.BackendError) as ei:
        sc.GgufModel(path)
    return ei.value


def qwen4exp_metadata():
    """The reference test's metadata set (reader_tests.rs:143-199)."""
    return [("general.architecture", STRING, "qwen4exp"), ("general.alignment", U32, 32),
            ("qwen4exp.block_count", U32, 48), ("qwen4exp.embedding_length", U32, 2560),
            ("qwen4exp.expert_count", U32, 512), ("qwen4exp.expert_used_count", U32, 10),
            ("qwen4exp.attention.head_count", U32, 24), ("qwen4exp.attention.head_count_kv", U32, 2),
            ("qwen4exp.attention.layer_norm_rms_epsilon", F32, 1e-6),
            ("qwen4exp.attention.compress_ratios", ARRAY, (I32, [4 if l % 4 == 3 else 0 for l in range(48)])),
            ("tokenizer.ggml.tokens", ARRAY, (STRING, ["<|endoftext|>", "hello", " world"])),
            ("tokenizer.ggml.model", STRING, "gpt2")]


# ---------------------------------------------------------------- the reference's reader tests

def test_reads_back_metadata_and_tensors(tmp_path):
    """reader_tests.rs:201-233."""
    blk = q8_0_block(0x4000, [5])  # d = 2.0
    data, _, _ = build(qwen4exp_metadata(), [("blk.0.attn_q.weight", [32], Q8_0, blk)])
    with sc.GgufModel(write(tmp_path, "read-back.gguf", data)) as f:
        assert f.shard(0)["version"] == 3
        assert f.get("general.architecture").as_str() == "qwen4exp"
        assert f.get("qwen4exp.block_count").as_int() == 48
        assert f.get("tokenizer.ggml.tokens").count == 3
        assert abs(f.get("qwen4exp.attention.layer_norm_rms_epsilon").as_float() - 1e-6) < 1e-12
        t = f.find("blk.0.attn_q.weight")
        assert t.shape == [32] and t.ty == Q8_0
        td = f.tensor_data("blk.0.attn_q.weight")
        assert td[2] == 5 and td.nbytes == 34
        assert oracle.dequantize_row(Q8_0, td, 32)[0] == 10.0


def test_bad_magic_is_refused(tmp_path):
    """reader_tests.rs:285-291."""
    e = open_err(write(tmp_path, "bad-magic.gguf", b"NOTGGUF and more bytes................"))
    assert e.code == sc.ERR_BAD_MAGIC and "bad magic 0x47544f4e" in str(e)  # "NOTG" read little-endian


def test_split_paths_resolves_siblings(tmp_path):
    """reader_tests.rs:293-300."""
    assert sc.split_paths("D:/models/qwen4exp-q2_0.gguf") == ["D:/models/qwen4exp-q2_0.gguf"]
    with pytest.raises(sc.BackendError) as ei:
        sc.split_paths("D:/nope/model-00001-of-00002.gguf")
    assert ei.value.code == sc.ERR_IO and "00002" in str(ei.value)
    assert "missing model shard 1 of 2 (is the download complete?)" in str(ei.value)


def test_multi_shard_model_reads_tensors_across_shards(tmp_path):
    """reader_tests.rs:302-333."""
    w1 = qwen4exp_metadata() + [("split.count", U32, 2), ("split.no", U32, 0), ("split.tensors.count", U32, 2)]
    d1, _, _ = build(w1, [("token_embd.weight", [32], F32_T, bytes(128))])
    w2 = [("split.count", U32, 2), ("split.no", U32, 1), ("split.tensors.count", U32, 2)]
    d2, _, _ = build(w2, [("output.weight", [32], F32_T, b"\x01" * 128)])
    p1 = write(tmp_path, "strata-rs-test-model-00001-of-00002.gguf", d1)
    p2 = write(tmp_path, "strata-rs-test-model-00002-of-00002.gguf", d2)
    with sc.GgufModel(p2) as m:
        assert m.n_shards() == 2
        assert m.get("general.architecture").as_str() == "qwen4exp"
        assert m.find("token_embd.weight") is not None and m.find("output.weight") is not None
        assert m.find("output.weight").shard == 1
        assert m.tensor_data("output.weight")[0] == 1
        assert m.shard(0)["path"] == str(p1) and m.shard(1)["path"] == str(p2)
    assert sc.split_paths(str(p1)) == [str(p1), str(p2)]


# ---------------------------------------------------------------- split_paths shapes

@pytest.mark.parametrize("name", ["m-00001-of-00002.bin", "m-0001-of-00002.gguf", "m-00001-of-0002.gguf",
                                  "m-0000a-of-00002.gguf", "m-00003-of-00002.gguf", "m-00000-of-00002.gguf",
                                  "m-00001-of-00000.gguf", "m_00001-of-00002.gguf", "00001-of-00002.gguf",
                                  "m-00001-of-00002.gguf.part"])
def test_split_paths_other_shapes_are_single_files(name):
    """Anything but `<stem>-NNNNN-of-MMMMM.gguf` with 1 <= N <= M is one file."""
    assert sc.split_paths("/x/" + name) == ["/x/" + name]


def test_split_paths_from_any_shard_lists_all_in_order(tmp_path):
    for i in range(1, 4):
        write(tmp_path, f"m-{i:05d}-of-00003.gguf", b"")
    want = [str(tmp_path / f"m-{i:05d}-of-00003.gguf") for i in range(1, 4)]
    for i in range(1, 4):
        assert sc.split_paths(str(tmp_path / f"m-{i:05d}-of-00003.gguf")) == want
    (tmp_path / "m-00002-of-00003.gguf").unlink()
    with pytest.raises(sc.BackendError) as ei:
        sc.split_paths(str(tmp_path / "m-00001-of-00003.gguf"))
    assert ei.value.code == sc.ERR_IO and "m-00002-of-00003.gguf" in str(ei.value)
    assert "missing model shard 2 of 3" in str(ei.value)


# ---------------------------------------------------------------- header checks

def valid_file():
    blk = q8_0_block(0x3C00, list(range(32)))
    return build([("general.architecture", STRING, "qwen4exp"), ("a.list", ARRAY, (U16, [1, 2, 3]))],
                 [("t0", [32, 2], Q8_0, blk * 2), ("t1", [64], Q8_0, blk * 2)])


def test_every_truncation_is_refused_or_bounds_checked(tmp_path):
    """Each prefix of a valid file: a header cut is Truncated at open; a data
    cut opens (the directory is whole) and the tensors past the end are
    Truncated when their payload is asked for."""
    data, data_start, offsets = valid_file()
    sizes = {"t0": 68, "t1": 68}
    p = tmp_path / "cut.gguf"
    for n in range(len(data)):
        p.write_bytes(data[:n])
        if n < data_start:
            e = open_err(p)
            assert e.code == sc.ERR_TRUNCATED, (n, e)
            continue
        with sc.GgufModel(p) as m:
            for (name, off) in zip(("t0", "t1"), offsets):
                end = data_start + off + sizes[name]
                if end <= n:
                    assert m.tensor_data(name).nbytes == sizes[name]
                else:
                    with pytest.raises(sc.BackendError) as ei:
                        m.tensor_data(name)
                    assert ei.value.code == sc.ERR_TRUNCATED
                    found = max(0, n - (data_start + off))
                    assert f"expected {sizes[name]} more bytes, found {found}" in str(ei.value)


def test_empty_and_missing_files(tmp_path):
    e = open_err(write(tmp_path, "empty.gguf", b""))
    assert e.code == sc.ERR_TRUNCATED and "expected 4 more bytes, found 0" in str(e)
    e = open_err(tmp_path / "nope.gguf")
    assert e.code == sc.ERR_IO and "No such file or directory (os error 2)" in str(e)
    e = open_err(tmp_path)
    assert e.code == sc.ERR_IO and "is a directory" in str(e)
    import os
    os.mkfifo(tmp_path / "fifo.gguf")  # refused at once, not waited on for a writer
    e = open_err(tmp_path / "fifo.gguf")
    assert e.code == sc.ERR_IO and "not a regular file" in str(e)


@pytest.mark.parametrize("version", [1, 2, 4])
def test_only_version_3_is_read(tmp_path, version):
    data, _, _ = build([], [], version=version)
    e = open_err(write(tmp_path, "v.gguf", data))
    assert e.code == sc.ERR_UNSUPPORTED_VERSION
    assert f"unsupported GGUF version {version} (expected 2 or 3)" in str(e)


def test_string_length_limit(tmp_path):
    ok, _, _ = build([("k" * 65535, U8, 1)])
    with sc.GgufModel(write(tmp_path, "ok.gguf", ok)) as m:
        assert m.get("k" * 65535).as_int() == 1
    raw = struct.pack("<Q", 65536) + b"k" * 65536 + struct.pack("<IB", U8, 1)
    bad, _, _ = build([], raw_kv=raw, n_kv=1)
    e = open_err(write(tmp_path, "long.gguf", bad))
    assert e.code == sc.ERR_BAD_KEY_LENGTH and "invalid metadata key length 65536 (max 65535)" in str(e)
    # string values have the same limit; the length alone is checked first
    raw = gstring("k") + struct.pack("<IQ", STRING, 1 << 40)
    bad, _, _ = build([], raw_kv=raw, n_kv=1)
    assert open_err(write(tmp_path, "longv.gguf", bad)).code == sc.ERR_BAD_KEY_LENGTH


@pytest.mark.parametrize("raw,ok", [(b"plain", True), ("é日本😀".encode(), True), (b"\xff", False),
                                    (b"\xc0\x80", False), (b"\xed\xa0\x80", False), (b"\xf4\x90\x80\x80", False),
                                    (b"\xe0\x80\x80", False), (b"\xe2\x82", False), (b"\x80", False),
                                    (b"\xf0\x90\x80\x80", True), (b"\xef\xbf\xbf", True), (b"\x00", True)])
def test_utf8_is_strict(tmp_path, raw, ok):
    data, _, _ = build([], raw_kv=gstring(raw) + struct.pack("<IB", U8, 7), n_kv=1)
    p = write(tmp_path, "u.gguf", data)
    if ok:
        with sc.GgufModel(p) as m:
            if b"\x00" in raw:  # a NUL is valid UTF-8, but C strings cannot name that key
                assert m.shard(0)["n_metadata"] == 1
            else:
                assert m.get(raw.decode()).as_int() == 7
    else:
        e = open_err(p)
        assert e.code == sc.ERR_STRING_NOT_UTF8 and "string is not valid UTF-8" in str(e)


def test_value_types(tmp_path):
    kvs = [("u8", U8, 255), ("i8", I8, -128), ("u16", U16, 65535), ("i16", I16, -32768), ("u32", U32, 2**32 - 1),
           ("i32", I32, -2**31), ("f32", F32, 1.5), ("b0", BOOL, 0), ("b1", BOOL, 1), ("s", STRING, "x"),
           ("u64", U64, 2**64 - 1), ("i64", I64, -2**63), ("f64", F64, -2.25),
           ("arr", ARRAY, (F64, [1.0, 2.0])), ("nest", ARRAY, (ARRAY, [(U8, [1, 2]), (U8, [])]))]
    data, _, _ = build(kvs)
    with sc.GgufModel(write(tmp_path, "types.gguf", data)) as m:
        assert m.shard(0)["n_metadata"] == len(kvs)
        want_int = {"u8": 255, "i8": -128, "u16": 65535, "i16": -32768, "u32": 2**32 - 1, "i32": -2**31, "b0": 0,
                    "b1": 1, "i64": -2**63}
        for k, v in want_int.items():
            assert m.get(k).as_int() == v, k
        assert m.get("u64").uint == 2**64 - 1 and m.get("u64").int == 0  # u64 payloads live apart
        assert m.get("f32").as_float() == 1.5 and m.get("f64").as_float() == -2.25 and m.get("f32").as_int() is None
        assert m.get("s").as_str() == "x" and m.get("s").as_int() is None
        assert m.get("arr").count == 2 and m.get("arr").elem == F64
        assert m.get("nest").count == 2 and m.get("nest").elem == ARRAY
        assert m.get("missing") is None


def test_a_later_duplicate_key_wins(tmp_path):
    data, _, _ = build([("k", U32, 1), ("k", U32, 2)])
    with sc.GgufModel(write(tmp_path, "dup.gguf", data)) as m:
        assert m.get("k").as_int() == 2 and m.shard(0)["n_metadata"] == 1


@pytest.mark.parametrize("raw,what", [
    (gstring("k") + struct.pack("<I", 13), "invalid metadata value type 13"),
    (gstring("k") + struct.pack("<IIQ", ARRAY, 99, 0), "invalid metadata value type 99"),
    (gstring("k") + struct.pack("<IIQ", ARRAY, U8, (1 << 24) + 1), "invalid metadata value type 9"),
    # arrays nest two deep at most: an array of arrays of arrays with an item is refused
    (gstring("k") + struct.pack("<IIQ", ARRAY, ARRAY, 1) + struct.pack("<IQ", ARRAY, 1) + struct.pack("<IQ", U8, 1)
     + b"\x01", "invalid metadata value type 9"),
])
def test_bad_value_types(tmp_path, raw, what):
    data, _, _ = build([], raw_kv=raw, n_kv=1)
    e = open_err(write(tmp_path, "vt.gguf", data))
    assert e.code == sc.ERR_BAD_VALUE_TYPE and what in str(e)


def test_array_limits(tmp_path):
    # three levels with empty innermost arrays parse (no item at depth 3 is read)
    raw = gstring("k") + struct.pack("<IIQ", ARRAY, ARRAY, 1) + struct.pack("<IQ", ARRAY, 1) + struct.pack("<IQ", U8, 0)
    data, _, _ = build([], raw_kv=raw, n_kv=1)
    with sc.GgufModel(write(tmp_path, "n.gguf", data)) as m:
        assert m.get("k").count == 1
    # exactly 2^24 items is allowed by the count check
    raw = gstring("k") + struct.pack("<IIQ", ARRAY, U8, 1 << 24) + bytes(64) + kv("next", U32, 9)
    data, _, _ = build([], raw_kv=raw, n_kv=2)
    with sc.GgufModel(write(tmp_path, "big.gguf", data)) as m:
        # arrays longer than 2^20 items have only their first 64 read through, as the
        # reference does (reader.rs:161-168), so the next key follows those 64 bytes
        assert m.get("k").count == 1 << 24 and m.get("next").as_int() == 9
    raw = gstring("k") + struct.pack("<IIQ", ARRAY, U8, 1 << 20) + bytes(1 << 20) + kv("next", U32, 9)
    data, _, _ = build([], raw_kv=raw, n_kv=2)
    with sc.GgufModel(write(tmp_path, "full.gguf", data)) as m:
        assert m.get("k").count == 1 << 20 and m.get("next").as_int() == 9


# ---------------------------------------------------------------- the tensor directory

def test_duplicate_tensor_names(tmp_path):
    blk = q8_0_block(0x3C00, [1])
    data, _, _ = build([], [("w", [32], Q8_0, blk), ("w", [32], Q8_0, blk)])
    e = open_err(write(tmp_path, "d.gguf", data))
    assert e.code == sc.ERR_TENSOR_NOT_FOUND and "tensor 'w' is missing from the file" in str(e)
    d1, _, _ = build([], [("w", [32], Q8_0, blk)])
    d2, _, _ = build([], [("w", [32], Q8_0, blk)])
    write(tmp_path, "m-00001-of-00002.gguf", d1)
    write(tmp_path, "m-00002-of-00002.gguf", d2)
    assert open_err(tmp_path / "m-00001-of-00002.gguf").code == sc.ERR_TENSOR_NOT_FOUND


@pytest.mark.parametrize("nd", [0, 5, 2**31])
def test_tensor_dims_1_to_4(tmp_path, nd):
    raw = gstring("w") + struct.pack("<I", nd)
    head = b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + raw
    e = open_err(write(tmp_path, "nd.gguf", head + bytes(64)))
    assert e.code == sc.ERR_WRONG_TENSOR_DIMS and f"tensor 'w' has {nd} dimensions, expected 4" in str(e)


def test_four_dims_read(tmp_path):
    blk = q8_0_block(0x3C00, [1])
    data, _, _ = build([], [("w", [32, 1, 1, 2], Q8_0, blk * 2)])
    with sc.GgufModel(write(tmp_path, "4d.gguf", data)) as m:
        assert m.find("w").shape == [32, 1, 1, 2] and m.tensor_data("w").nbytes == 68


# ---------------------------------------------------------------- alignment and the data start

@pytest.mark.parametrize("ty,val,want", [(U32, 64, 64), (U8, 1, 1), (I64, 4096, 4096), (BOOL, 1, 1), (I32, -8, 32),
                                         (U32, 0, 32), (U64, 64, 32), (F32, 64.0, 32), (STRING, "64", 32)])
def test_alignment_from_metadata(tmp_path, ty, val, want):
    """general.alignment counts when MetaValue::as_int gives a positive value:
    a u64 keeps its payload outside `int` and so leaves the default 32."""
    blk = q8_0_block(0x3C00, [3])
    data, data_start, _ = build([("general.alignment", ty, val)], [("w", [32], Q8_0, blk)], align=want)
    with sc.GgufModel(write(tmp_path, "al.gguf", data)) as m:
        s = m.shard(0)
        assert s["alignment"] == want and s["data_start"] == data_start and data_start % want == 0
        assert m.tensor_data("w")[2] == 3


def test_metadata_only_shard_may_end_before_the_data_start(tmp_path):
    data, data_start, _ = build([("split.no", U32, 0)], [], pad=False)
    assert len(data) < data_start
    with sc.GgufModel(write(tmp_path, "meta.gguf", data)) as m:
        assert m.shard(0)["data_start"] == len(data) and m.tensor_count() == 0


def test_a_shard_with_tensors_must_reach_the_data_start(tmp_path):
    blk = q8_0_block(0x3C00, [1])
    data, data_start, _ = build([], [("w", [32], Q8_0, blk)])
    head_end = data_start - 1
    e = open_err(write(tmp_path, "short.gguf", data[:head_end]))
    assert e.code == sc.ERR_TRUNCATED and f"expected {data_start} more bytes, found {head_end}" in str(e)


# ---------------------------------------------------------------- payloads

def test_payload_checks(tmp_path):
    blk = q8_0_block(0x3C00, [1])
    tensors = [("zero", [32, 0], Q8_0, b""), ("unknown", [32], 99, blk), ("huge", [2**40, 2**40], Q8_0, b""),
               ("wrap", [2**63, 4], F32_T, b""), ("ok", [32], Q8_0, blk), ("partial", [33], Q8_0, blk),
               ("past", [64], Q8_0, blk)]
    data, data_start, offsets = build([], tensors)
    with sc.GgufModel(write(tmp_path, "pay.gguf", data)) as m:
        def err(name):
            with pytest.raises(sc.BackendError) as ei:
                m.tensor_data(name)
            return ei.value
        e = err("zero")
        assert e.code == sc.ERR_TRUNCATED and f"expected {offsets[0]} more bytes, found 0" in str(e)
        e = err("unknown")
        assert e.code == sc.ERR_UNSUPPORTED_QUANT and 'unsupported quantization type "type id 99"' in str(e)
        assert err("huge").code == sc.ERR_TRUNCATED
        assert err("wrap").code == sc.ERR_TRUNCATED  # 2^65 elements: the product overflows
        assert m.tensor_data("ok").nbytes == 34
        # a row that is not whole blocks: the payload counts whole blocks only, as tensor_payload_bytes
        assert m.tensor_data("partial").nbytes == 34
        # the last tensor needs 2 blocks and the file holds 1
        e = err("past")
        assert e.code == sc.ERR_TRUNCATED and "expected 68 more bytes, found 34" in str(e)


@pytest.mark.parametrize("off", ["eof", 2**64 - 1, 2**64 - 16])
def test_payload_offsets_past_the_end_or_overflowing(tmp_path, off):
    blk = q8_0_block(0x3C00, [1])
    data, data_start, _ = build([], [("w", [32], Q8_0, blk)])
    off = len(data) - data_start if off == "eof" else off
    at = 24 + len(tensor_info("w", [32], Q8_0, 0)) - 8  # the directory entry's offset field
    raw = data[:at] + struct.pack("<Q", off) + data[at + 8:]
    with sc.GgufModel(write(tmp_path, "off.gguf", raw)) as m:
        assert m.find("w").offset == off
        with pytest.raises(sc.BackendError) as ei:
            m.tensor_data("w")
        assert ei.value.code == sc.ERR_TRUNCATED


def test_random_models_round_trip(tmp_path):
    """Random directories: the reader reports each tensor's shape, type, offset
    and exactly its bytes, across shards."""
    g = rng(5150)
    types = [sc.Q8_0, sc.Q4_K, sc.Q5_K, sc.Q6_K, sc.Q4_0, sc.F32, sc.F16, sc.BF16, sc.IQ4_XS, sc.MXFP4]
    for it in range(6):
        n_shards = 1 + it % 3
        expect = {}
        for s in range(n_shards):
            tensors = []
            for k in range(int(g.integers(0, 6))):
                ty = types[int(g.integers(len(types)))]
                bs, ts = sc.BLOCK[ty]
                nd = int(g.integers(1, 4))
                shape = [bs * int(g.integers(1, 4))] + [int(g.integers(1, 4)) for _ in range(nd - 1)]
                nb = int(np.prod(shape)) // bs
                blob = g.integers(0, 256, nb * ts, dtype=np.uint8).tobytes()
                name = f"s{s}.t{k}"
                tensors.append((name, shape, ty, blob))
                expect[name] = (shape, ty, blob, s)
            al = [32, 64, 1, 256][it % 4]
            kvs = [("general.alignment", U32, al), ("rand", U64, int(g.integers(0, 2**62)))]
            data, _, offsets = build(kvs, tensors, align=al, data_align=al)
            name = f"r{it}-{s + 1:05d}-of-{n_shards:05d}.gguf" if n_shards > 1 else f"r{it}.gguf"
            write(tmp_path, name, data)
        path = tmp_path / (f"r{it}-00001-of-{n_shards:05d}.gguf" if n_shards > 1 else f"r{it}.gguf")
        with sc.GgufModel(path) as m:
            assert m.n_shards() == n_shards and m.tensor_count() == len(expect)
            names = [t.name for t in m.tensors()]
            assert names == list(expect)
            for nm, (shape, ty, blob, s) in expect.items():
                t = m.find(nm)
                assert (t.shape, t.ty, t.shard) == (shape, ty, s)
                assert m.tensor_data(nm).tobytes() == blob


def test_null_arguments_are_refused():
    L = sc.lib()
    assert L.strata_cuda_gguf_open(None, None, None, 0) == sc.ERR_INVALID
    assert L.strata_cuda_gguf_tensor_count(None) == 0
    assert L.strata_cuda_gguf_n_shards(None) == 0
    assert L.strata_cuda_gguf_ingest(None, None, None, 0, None) == sc.ERR_INVALID
    assert L.strata_cuda_upload_many(None, None, 0, None) == sc.ERR_INVALID
    L.strata_cuda_gguf_close(None)


# ---------------------------------------------------------------- views: what one rank reads

def view_bytes(v) -> bytes:
    import ctypes
    return ctypes.string_at(v.bytes, v.len) if v.len else b""


def test_views_of_rows_and_experts(tmp_path):
    """strata_cuda_gguf_view: WeightStore's geometry (1-D one row, 2-D [cols, rows],
    3-D [cols, rows, n_expert]) and the byte slice of a row or expert range."""
    g = rng(808)
    dense = g.integers(0, 256, 12 * 2 * 144, dtype=np.uint8).tobytes()    # Q4_K [512, 12]
    experts = g.integers(0, 256, 5 * 4 * 34, dtype=np.uint8).tobytes()    # Q8_0 [32, 4, 5]
    norm = g.integers(0, 256, 64 * 4, dtype=np.uint8).tobytes()           # F32 [64]
    data, _, _ = build([], [("dense", [512, 12], Q4_K, dense), ("exps", [32, 4, 5], Q8_0, experts),
                            ("norm", [64], F32_T, norm), ("four", [32, 1, 1, 2], Q8_0, bytes(68)),
                            ("ragged", [33, 2], Q8_0, bytes(68))])
    with sc.GgufModel(write(tmp_path, "views.gguf", data)) as m:
        v = m.view("dense")
        assert (v.quant, v.n_expert, v.rows, v.cols, v.len) == (Q4_K, 0, 12, 512, len(dense))
        assert view_bytes(v) == dense
        v = m.view("dense", 3, 4)
        assert (v.rows, v.cols, v.n_expert) == (4, 512, 0) and view_bytes(v) == dense[3 * 288:7 * 288]
        v = m.view("dense", 12, 0)
        assert v.len == 0 and v.rows == 0
        v = m.view("exps")
        assert (v.quant, v.n_expert, v.rows, v.cols) == (Q8_0, 5, 4, 32) and view_bytes(v) == experts
        v = m.view("exps", 2, -1)
        assert (v.n_expert, v.rows) == (3, 4) and view_bytes(v) == experts[2 * 136:]
        v = m.view("norm")
        assert (v.quant, v.n_expert, v.rows, v.cols) == (F32_T, 0, 1, 64) and view_bytes(v) == norm
        for name, first, count in [("dense", 0, 13), ("dense", 13, 0), ("dense", -1, 2), ("exps", 4, 2),
                                   ("norm", 1, 1), ("four", 0, -1)]:
            with pytest.raises(sc.BackendError) as ei:
                m.view(name, first, count)
            assert ei.value.code == sc.ERR_INVALID, (name, first, count)
        with pytest.raises(sc.BackendError) as ei:  # rows that are not whole blocks
            m.view("ragged")
        assert ei.value.code == sc.ERR_TRUNCATED


def test_shard_views_cover_the_tensor_once(tmp_path):
    """Each rank's row or expert range (strata-rs_b200/sharding.py): the ranks'
    slices are disjoint, in order, and together the whole payload."""
    import sharding
    g = rng(909)
    dense = g.integers(0, 256, 64 * 8 * 144, dtype=np.uint8).tobytes()    # Q4_K [2048, 64]
    experts = g.integers(0, 256, 16 * 8 * 288, dtype=np.uint8).tobytes()  # Q4_K [512, 8, 16]
    data, _, _ = build([], [("proj", [2048, 64], Q4_K, dense), ("exps", [512, 8, 16], Q4_K, experts)])
    with sc.GgufModel(write(tmp_path, "shards.gguf", data)) as m:
        for world in (1, 2, 4, 8):
            rows = [sharding.row_shard_view(m, "proj", world, r) for r in range(world)]
            assert b"".join(view_bytes(v) for v in rows) == dense
            assert all(v.rows == 64 // world and v.n_expert == 0 for v in rows)
            exps = [sharding.expert_shard_view(m, "exps", world, r) for r in range(world)]
            assert b"".join(view_bytes(v) for v in exps) == experts
            assert all(v.n_expert == 16 // world and v.rows == 8 and v.cols == 512 for v in exps)
