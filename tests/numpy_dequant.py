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


DEQUANT = {8: q8_0, 12: q4_k, 13: q5_k, 14: q6_k}
