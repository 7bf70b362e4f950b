"""Seeded synthetic weights and activations for the benchmark configs.

The reference publishes no benchmark data, so every input is generated here
from a fixed numpy PCG64 seed with the shapes and value distributions the
benchmark configs name:

* Q8_0: fp16 d ~ U(0.002, 0.02), 32 int8 quants uniform in [-127, 127].
* Q4_K / Q5_K: random block bytes, then fp16 d and dmin ~ U(0.001, 0.01).
* Q6_K: random block bytes, then fp16 d (at byte 208) ~ U(0.001, 0.01); the
  16 scales stay random u8 (strata reads them unsigned).
* activations: standard normal f32; bf16 inputs are the RNE rounding of those.

Blocks are laid out exactly as strata-gguf stores them (row-major rows, each
row a run of blocks), so the arrays upload byte-for-byte.
"""
from __future__ import annotations

import numpy as np

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 8, 12, 13, 14, 30
# the other block formats (crates/strata-gguf/src/quant.rs:15-43, 124-163)
Q4_0, Q4_1, Q5_0, Q5_1, Q8_1, Q2_K, Q3_K, IQ4_NL, IQ4_XS, MXFP4, NVFP4, Q2_0 = 2, 3, 6, 7, 9, 10, 11, 20, 23, 39, 40, 42
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176),
         Q6_K: (256, 210), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), Q8_1: (32, 36),
         Q2_K: (256, 84), Q3_K: (256, 110), IQ4_NL: (32, 18), IQ4_XS: (256, 136), MXFP4: (32, 17),
         NVFP4: (64, 36), Q2_0: (64, 18)}
OTHER_FORMATS = [Q4_0, Q4_1, Q5_0, Q5_1, Q8_1, Q2_K, Q3_K, IQ4_NL, IQ4_XS, MXFP4, NVFP4, Q2_0]


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _f16(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint16)


def quant_blocks(g: np.random.Generator, quant: int, n_blocks: int,
                 d_range: tuple[float, float] | None = None) -> np.ndarray:
    """n_blocks random blocks of `quant` as a (n_blocks, type_size) uint8 array."""
    bs, ts = BLOCK[quant]
    if quant in (F32, F16, BF16):
        vals = g.standard_normal(n_blocks).astype(np.float32)
        if quant == F32:
            return vals.view(np.uint8).reshape(n_blocks, 4)
        if quant == F16:
            return _f16(vals).view(np.uint8).reshape(n_blocks, 2)
        return bf16_bits(vals).view(np.uint8).reshape(n_blocks, 2)
    b = g.integers(0, 256, size=(n_blocks, ts), dtype=np.uint8)
    if quant == Q8_0:
        lo, hi = d_range or (0.002, 0.02)
        b[:, 0:2] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
        b[:, 2:34] = g.integers(-127, 128, size=(n_blocks, 32), dtype=np.int8).view(np.uint8)
    elif quant in (Q4_K, Q5_K):
        lo, hi = d_range or (0.001, 0.01)
        b[:, 0:2] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
        b[:, 2:4] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
    elif quant == Q6_K:
        lo, hi = d_range or (0.001, 0.01)
        b[:, 208:210] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
    elif quant in (Q4_1, Q5_1, Q2_K):
        # fp16 d and a second fp16 (min / dmin) at byte 2
        lo, hi = d_range or (0.001, 0.01)
        b[:, 0:2] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
        b[:, 2:4] = _f16(g.uniform(-hi, hi, n_blocks) if quant != Q2_K else g.uniform(lo, hi, n_blocks)) \
            .view(np.uint8).reshape(n_blocks, 2)
    elif quant == Q3_K:
        lo, hi = d_range or (0.001, 0.01)
        b[:, 108:110] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
    elif quant == MXFP4:
        b[:, 0] = g.integers(110, 125, size=n_blocks)          # E8M0 2^-17 .. 2^-3
    elif quant == NVFP4:
        b[:, 0:4] = g.integers(0x18, 0x48, size=(n_blocks, 4))  # UE4M3 ~2^-4 .. 2^2, finite
    elif quant in (Q4_0, Q5_0, Q8_1, IQ4_NL, IQ4_XS, Q2_0):
        lo, hi = d_range or (0.001, 0.01)
        b[:, 0:2] = _f16(g.uniform(lo, hi, n_blocks)).view(np.uint8).reshape(n_blocks, 2)
    return b


def quant_matrix(seed: int, quant: int, rows: int, cols: int, n_expert: int = 0) -> np.ndarray:
    """A [n_expert or 1][rows][cols] tensor of `quant` as flat uint8 bytes."""
    bs, ts = BLOCK[quant]
    assert cols % bs == 0
    mats = max(1, n_expert)
    nb = mats * rows * (cols // bs)
    return quant_blocks(rng(seed), quant, nb).reshape(-1)


def activations(seed: int, batch: int, k: int) -> np.ndarray:
    return rng(seed).standard_normal((batch, k)).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits, round half to even (half::bf16::from_f32, finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)


# The benchmark configs (K -> N). Q4_K decode sweep shapes (the headline workload):
Q4K_SWEEP = [(4096, 4096), (4096, 12288), (12288, 4096), (2048, 151936)]
SWEEP_BATCHES = [1, 2, 4, 8]
