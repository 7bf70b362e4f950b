"""A second, independent restatement of the four block formats, vectorised
over all blocks with numpy, written from the byte layouts rather than from the
scalar loops. Tests compare it with the C oracle bit for bit, which guards the
oracle against transcription slips (the reference's own tests pin only Q8_0
and Q6_K by known answers: crates/strata-gguf/tests/dequant_tests.rs:71-79,160-169).

float32 numpy arithmetic rounds every operation, like Rust without FMA.
"""
import numpy as np

f32 = np.float32


def _f16(b2: np.ndarray) -> np.ndarray:
    return b2.copy().view(np.float16).astype(np.float32).reshape(-1)


def _scale_min(sc12: np.ndarray):
    """(n, 12) scale bytes -> sc (n, 8), m (n, 8) as uint8 (get_scale_min_k4)."""
    q = sc12.astype(np.uint8)
    sc = np.empty((q.shape[0], 8), np.uint8)
    m = np.empty((q.shape[0], 8), np.uint8)
    sc[:, :4] = q[:, 0:4] & 63
    m[:, :4] = q[:, 4:8] & 63
    sc[:, 4:] = (q[:, 8:12] & 0x0F) | ((q[:, 0:4] >> 6) << 4)
    m[:, 4:] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return sc, m


def q8_0(blocks: np.ndarray) -> np.ndarray:
    d = _f16(blocks[:, 0:2])
    q = blocks[:, 2:34].view(np.int8).astype(np.float32)
    return (q * d[:, None]).astype(f32).reshape(-1)


def _k4(blocks, d, dm, sc12, q_lo, q_hi):
    """q_lo/q_hi: (n, 8, 32) 0..31 values per sub-block; returns (n, 256)."""
    sc, m = _scale_min(sc12)
    d1 = (d[:, None] * sc.astype(f32)).astype(f32)      # (n, 8)
    m1 = (dm[:, None] * m.astype(f32)).astype(f32)
    out = (d1[:, :, None] * q_lo.astype(f32)).astype(f32) - m1[:, :, None]
    return out.astype(f32).reshape(blocks.shape[0], 256)


def q4_k(blocks: np.ndarray) -> np.ndarray:
    n = blocks.shape[0]
    d, dm = _f16(blocks[:, 0:2]), _f16(blocks[:, 2:4])
    qs = blocks[:, 16:144].reshape(n, 4, 32)
    vals = np.empty((n, 8, 32), np.uint8)
    vals[:, 0::2] = qs & 0x0F   # sub-block 2c: low nibbles of chunk c
    vals[:, 1::2] = qs >> 4     # sub-block 2c+1: high nibbles
    return _k4(blocks, d, dm, blocks[:, 4:16], vals, None).reshape(-1)


def q5_k(blocks: np.ndarray) -> np.ndarray:
    n = blocks.shape[0]
    d, dm = _f16(blocks[:, 0:2]), _f16(blocks[:, 2:4])
    qh = blocks[:, 16:48]                     # (n, 32)
    qs = blocks[:, 48:176].reshape(n, 4, 32)
    vals = np.empty((n, 8, 32), np.uint8)
    for j in range(8):
        nib = (qs[:, j // 2] & 0x0F) if j % 2 == 0 else (qs[:, j // 2] >> 4)
        vals[:, j] = nib + 16 * ((qh >> j) & 1)
    return _k4(blocks, d, dm, blocks[:, 4:16], vals, None).reshape(-1)


def q6_k(blocks: np.ndarray) -> np.ndarray:
    n = blocks.shape[0]
    ql = blocks[:, 0:128].reshape(n, 2, 64)
    qh = blocks[:, 128:192].reshape(n, 2, 32)
    sc = blocks[:, 192:208].reshape(n, 2, 8).astype(f32)   # u8 scales
    d = _f16(blocks[:, 208:210])
    out = np.empty((n, 2, 4, 32), f32)
    for g in range(4):                       # quarter g of each 128-half
        src = ql[:, :, 0:32] if g in (0, 2) else ql[:, :, 32:64]
        nib = (src & 0x0F) if g < 2 else (src >> 4)
        q = (nib | (((qh >> (2 * g)) & 3) << 4)).astype(np.int32) - 32
        s = np.repeat(sc[:, :, 2 * g:2 * g + 2], 16, axis=2)    # is = l // 16
        out[:, :, g] = ((d[:, None, None] * s).astype(f32) * q.astype(f32)).astype(f32)
    return out.reshape(-1)


# ---- the other block formats, from their byte layouts


def _nibbles(qs: np.ndarray) -> np.ndarray:
    """(n, 16) bytes -> (n, 32) values: low nibbles first, then high (elements j, j + 16)."""
    return np.concatenate([qs & 0x0F, qs >> 4], axis=1)


def _bits32(b4: np.ndarray) -> np.ndarray:
    """(n, 4) little-endian bytes -> (n, 32) bits, bit i at column i."""
    w = b4.copy().view(np.uint32).reshape(-1)
    return ((w[:, None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.uint8)


def q4_0(b):
    return (((_nibbles(b[:, 2:18]).astype(f32) - f32(8)).astype(f32)) * _f16(b[:, 0:2])[:, None]).astype(f32).reshape(-1)


def q4_1(b):
    d, m = _f16(b[:, 0:2])[:, None], _f16(b[:, 2:4])[:, None]
    return ((_nibbles(b[:, 4:20]).astype(f32) * d).astype(f32) + m).astype(f32).reshape(-1)


def q5_0(b):
    x = _nibbles(b[:, 6:22]) | (_bits32(b[:, 2:6]) << 4)
    return (((x.astype(f32) - f32(16)).astype(f32)) * _f16(b[:, 0:2])[:, None]).astype(f32).reshape(-1)


def q5_1(b):
    d, m = _f16(b[:, 0:2])[:, None], _f16(b[:, 2:4])[:, None]
    x = _nibbles(b[:, 8:24]) | (_bits32(b[:, 4:8]) << 4)
    return ((x.astype(f32) * d).astype(f32) + m).astype(f32).reshape(-1)


def q8_1(b):
    return (b[:, 4:36].view(np.int8).astype(f32) * _f16(b[:, 0:2])[:, None]).astype(f32).reshape(-1)


def q2_0(b):
    codes = ((b[:, 2:18, None] >> (2 * np.arange(4, dtype=np.uint8))) & 3).reshape(-1, 64)
    return (((codes.astype(f32) - f32(1)).astype(f32)) * _f16(b[:, 0:2])[:, None]).astype(f32).reshape(-1)


IQ4 = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.int8)


def iq4_nl(b):
    return (_f16(b[:, 0:2])[:, None] * IQ4[_nibbles(b[:, 2:18])].astype(f32)).astype(f32).reshape(-1)


def iq4_xs(b):
    n = b.shape[0]
    d = _f16(b[:, 0:2])
    sh = b[:, 2:4].copy().view(np.uint16).reshape(-1).astype(np.uint32)
    ib = np.arange(8)
    ls = ((b[:, 4 + ib // 2] >> (4 * (ib % 2))) & 0x0F).astype(np.uint32) | (((sh[:, None] >> (2 * ib)) & 3) << 4)
    dl = (d[:, None] * (ls.astype(f32) - f32(32)).astype(f32)).astype(f32)          # (n, 8)
    # strata-gguf's dequant_iq4_xs reads qs[0..16] for every sub-block (dequant.rs:194-203)
    vals = IQ4[_nibbles(b[:, 8:24])].astype(f32)                                        # (n, 32)
    return (dl[:, :, None] * vals[:, None, :]).astype(f32).reshape(-1)


def q2_k(b):
    n = b.shape[0]
    d, mn = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    sc, q = b[:, 4:20], b[:, 20:84].reshape(n, 2, 32)
    out = np.empty((n, 2, 4, 32), f32)
    for g in range(2):
        s = (sc[:, 2 * g:2 * g + 2] & 63).astype(f32)          # is = 2g, 2g + 1 (j < 4)
        m = (sc[:, 2 * g + 4:2 * g + 6] & 63).astype(f32)
        dd = (d[:, None] * s).astype(f32)
        mm = (mn[:, None] * m).astype(f32)
        for f in range(4):                                     # 2-bit field f: sub-block f % 2
            v = ((q[:, g] >> (2 * f)) & 3).astype(f32)
            out[:, g, f] = ((dd[:, f % 2, None] * v).astype(f32) - mm[:, f % 2, None]).astype(f32)
    return out.reshape(-1)


def q3_k(b):
    n = b.shape[0]
    hm, q = b[:, 0:32], b[:, 32:96].reshape(n, 2, 32)
    d = _f16(b[:, 108:110])
    raw = b[:, 96:108]
    # 16 six-bit scales: low 4 bits from bytes 0..7 (nibbles), high 2 bits from bytes 8..11
    lo = np.concatenate([raw[:, 0:8] & 0x0F, raw[:, 0:8] >> 4], axis=1)            # scale i: i < 8 low, else high
    hi = ((raw[:, 8:12, None] >> (2 * np.arange(4, dtype=np.uint8))) & 3)           # (n, 4, 4): byte k, pair p
    hi = hi.transpose(0, 2, 1).reshape(n, 16)                                       # scale 4p + k
    sc = (lo | (hi << 4)).astype(np.int32) - 32
    out = np.empty((n, 2, 4, 2, 16), f32)
    for h in range(2):
        for s4 in range(4):
            bit = ((hm >> (4 * h + s4)) & 1).reshape(n, 2, 16)
            v = ((q[:, h] >> (2 * s4)) & 3).reshape(n, 2, 16).astype(f32)
            v = (v - np.where(bit == 1, f32(0), f32(4))).astype(f32)
            dl = (d[:, None] * sc[:, 8 * h + 2 * s4:8 * h + 2 * s4 + 2].astype(f32)).astype(f32)
            out[:, h, s4] = (dl[:, :, None] * v).astype(f32)
    return out.reshape(-1)


def _fp4(codes):
    mag = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], f32)[codes & 7]
    return np.where((codes & 8) != 0, -mag, mag).astype(f32) + f32(0)  # +0 for code 8


def mxfp4(b):
    e = b[:, 0].astype(np.uint32)
    d = np.where(e == 0, f32(0), (e << 23).view(np.float32)).astype(f32)
    return ((d[:, None] * (_fp4(_nibbles(b[:, 1:17])) * f32(2)).astype(f32)).astype(f32) * f32(0.5)).astype(f32).reshape(-1)


def nvfp4(b):
    n = b.shape[0]
    e = b[:, 0:4].astype(np.int32)
    ex, man = (e >> 3) & 15, e & 7
    v = np.where(ex == 0, (man.astype(f32) / f32(8)).astype(f32) * f32(2.0 ** -6),
                 np.ldexp(f32(1), ex - 7).astype(f32) * (f32(1) + (man.astype(f32) / f32(8)).astype(f32)))
    ds = np.where((e & 0x80) != 0, -v, v).astype(f32)                                 # (n, 4)
    qs = b[:, 4:36].reshape(n, 4, 8)
    vals = np.concatenate([qs & 0x0F, qs >> 4], axis=2)                                 # (n, 4, 16)
    return ((ds[:, :, None] * (_fp4(vals) * f32(2)).astype(f32)).astype(f32) * f32(0.5)).astype(f32).reshape(-1)


DEQUANT = {8: q8_0, 12: q4_k, 13: q5_k, 14: q6_k, 2: q4_0, 3: q4_1, 6: q5_0, 7: q5_1, 9: q8_1, 10: q2_k,
           11: q3_k, 20: iq4_nl, 23: iq4_xs, 39: mxfp4, 40: nvfp4, 42: q2_0}
