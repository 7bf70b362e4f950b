"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a machine without a GPU (oracle pins, host logic, the
C ABI's exports). `-m gpu` runs the parity tests proper on a B200: CUDA path
through the C ABI versus the CPU oracle on the same seeded inputs.
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "strata-rs_b200", ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max_i |y - ref| / max(|ref_i|, 1e-3 * ||ref||_inf): the parity metric for
    GEMV/GEMM outputs (near-zero outputs are judged against the vector's scale).
    The floor is taken per output vector: along the last axis, so each row of a
    batched output (one token's projection) is judged against its own norm."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return 0.0
    if ref.ndim == 0:
        ref, y = ref.reshape(1), y.reshape(1)
    floor = 1e-3 * np.maximum(np.max(np.abs(ref), axis=-1, keepdims=True), 1e-30)
    return float(np.max(np.abs(y - ref) / np.maximum(np.abs(ref), floor)))


@pytest.fixture(scope="session")
def threads():
    return max(1, os.cpu_count() or 1)
