"""A small GGUF v3 writer for the tests (test infrastructure, not product).

Builds files the way the GGUF layout defines them (crates/strata-gguf/src/
reader.rs:1-12): magic, version, counts, key/value metadata, the tensor
directory, padding to the alignment, then the tensor data at the directory's
offsets. Every field can be overridden so tests can write broken files too.
"""
from __future__ import annotations

import struct

# metadata value types (crates/strata-gguf/src/metadata.rs:11-27)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}


def gstring(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def payload(ty: int, v) -> bytes:
    """A value's bytes without its type tag (array items carry none)."""
    if ty == STRING:
        return gstring(v)
    if ty == ARRAY:
        elem, items = v
        return struct.pack("<IQ", elem, len(items)) + b"".join(payload(elem, it) for it in items)
    return struct.pack(_SCALAR[ty], v)


def kv(key, ty: int, v) -> bytes:
    return gstring(key) + struct.pack("<I", ty) + payload(ty, v)


def tensor_info(name, shape, ty: int, offset: int) -> bytes:
    return gstring(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape) + \
        struct.pack("<IQ", ty, offset)


def build(kvs=(), tensors=(), *, version: int = 3, magic: bytes = b"GGUF", align: int = 32, data_align: int = 32,
          raw_kv: bytes | None = None, n_kv: int | None = None, n_tensors: int | None = None,
          pad: bool = True):
    """Returns (file bytes, data_start, offsets).

    kvs: (key, type, value) triples; tensors: (name, shape, type, data bytes)
    with each tensor's data placed at the next multiple of `data_align` in the
    data section. `raw_kv` replaces the encoded metadata; `n_kv` / `n_tensors`
    override the header counts; `pad=False` ends the file right after the
    directory when there is no tensor data.
    """
    kv_bytes = raw_kv if raw_kv is not None else b"".join(kv(k, t, v) for k, t, v in kvs)
    offsets, data, off = [], b"", 0
    for _, _, _, blob in tensors:
        off = -(-off // data_align) * data_align
        data += b"\0" * (off - len(data)) + bytes(blob)
        offsets.append(off)
        off += len(blob)
    dir_bytes = b"".join(tensor_info(n, s, t, o) for (n, s, t, _), o in zip(tensors, offsets))
    head = magic + struct.pack("<IQQ", version, len(tensors) if n_tensors is None else n_tensors,
                               len(kvs) if n_kv is None else n_kv) + kv_bytes + dir_bytes
    data_start = -(-len(head) // align) * align
    if not pad and not data:
        return head, data_start, offsets
    return head + b"\0" * (data_start - len(head)) + data, data_start, offsets


def q8_0_block(d_bits: int, qs) -> bytes:
    """One Q8_0 block: fp16 scale bits, 32 int8 quants."""
    q = list(qs) + [0] * (32 - len(qs))
    return struct.pack("<H", d_bits) + struct.pack("<32b", *q)
