"""Builds the inputs of tests/golden/reference_kats.json (the reference's own
known-answer cases) as numpy arrays, shared by the CPU and GPU tests."""
import json
from pathlib import Path

import numpy as np

KATS = json.loads((Path(__file__).with_name("reference_kats.json")).read_text())


def f16_bytes(v: float) -> np.ndarray:
    return np.array([v], np.float16).view(np.uint8)


def dequant_case(case: dict) -> np.ndarray:
    b = np.zeros(case["block_len"], np.uint8)
    for off, v in case.get("set_f16", []):
        b[off:off + 2] = f16_bytes(v)
    for off, v in case.get("set_bytes", []):
        b[off] = v
    return b


def q2_0_invariant_block() -> np.ndarray:
    """dequant_tests.rs:43-60 (q2_0_structural_invariant): d = 0.5 and bytes
    (37 i + 11) mod 256; every output must be one of -d, 0, +d, +2d."""
    b = np.zeros(18, np.uint8)
    b[0:2] = f16_bytes(0.5)
    b[2:] = [(i * 37 + 11) & 0xFF for i in range(16)]
    return b


def lcg_block(quant: int, nbytes: int, spec: dict) -> np.ndarray:
    """dequant_tests.rs:219-237: LCG bytes, then a finite scale: the E8M0 /
    UE4M3 scale bytes of MXFP4 / NVFP4, an fp16 0.125 in the first two bytes
    of every other quantized type."""
    state = spec["seed"]
    out = np.empty(nbytes, np.uint8)
    for i in range(nbytes):
        state = (state * spec["mul"] + spec["add"]) & 0xFFFFFFFF
        out[i] = (state >> spec["shift"]) & 0xFF
    special = spec.get("scale_bytes", {}).get(str(quant))
    if special:
        for off, v in special:
            out[off] = v
    elif quant not in (0, 1, 30):
        out[0:2] = f16_bytes(spec["scale_f16"])
    return out


def gemv_case(case: dict):
    """(quant, weight bytes, rows, cols, x) of a gemv known-answer case."""
    q, rows, cols = case["quant"], case["rows"], case["cols"]
    if q == 8:
        block = np.zeros(34, np.uint8)
        block[0:2] = f16_bytes(case["d"])
        block[2:34] = np.array([(j % 7) - 3 for j in range(32)], np.int8).view(np.uint8)
        x = np.array([i * 0.25 - 1.0 for i in range(32)], np.float32)
        return q, block, rows, cols, x
    if q == 30:
        w = np.array(case["w_f32"], np.float32)
        from synth import bf16_bits
        return q, bf16_bits(w).view(np.uint8).copy(), rows, cols, np.array(case["x"], np.float32)
    r = np.arange(rows)[:, None]
    c = np.arange(cols)[None, :]
    if case["name"].startswith("gemv_matches_manual_dot"):
        w = (r * cols + c + 1).astype(np.float32)
        x = np.array(case["x"], np.float32)
    else:
        w = (((r * 7 + c) % 11) * 0.25 - 1.0).astype(np.float32)
        x = np.array([(i % 5) * 0.5 - 1.0 for i in range(cols)], np.float32)
    return q, w.reshape(-1).view(np.uint8).copy(), rows, cols, x


def expert_case(case: dict):
    E, rows, cols = case["n_expert"], case["rows"], case["cols"]
    e = np.arange(E)[:, None, None]
    r = np.arange(rows)[None, :, None]
    c = np.arange(cols)[None, None, :]
    w = (((e * 100 + r * 10 + c) % 13) * 0.2 - 1.0).astype(np.float32)
    x = np.array([(i % 3) - 0.5 for i in range(rows)], np.float32)
    return case["quant"], w.reshape(-1).view(np.uint8).copy(), E, rows, cols, x
