"""Mutation fuzzing of the GGUF reader on the CPU: strata-rs_b200/csrc/gguf.cpp
compiled with address and undefined-behaviour checks into tests/gguf_fuzz.cpp,
run over thousands of mutated copies of valid files. A model file is input
from outside; whatever its bytes, the reader must open it or refuse it,
never read outside the mapping."""
import shutil
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

import strata_cuda as sc
from gguf_writer import ARRAY, F32, I32, STRING, U8, U16, U32, U64, build, q8_0_block
from synth import rng

ROOT = Path(__file__).resolve().parents[1]
CUDA_INC = Path("/usr/local/cuda/include")


def seeds():
    g = rng(31337)
    blk = q8_0_block(0x3C00, list(range(32)))
    meta = [("general.architecture", STRING, "qwen35moe"), ("general.alignment", U32, 32),
            ("a.list", ARRAY, (U16, [1, 2, 3])), ("tokens", ARRAY, (STRING, ["a", "bc", ""])),
            ("nest", ARRAY, (ARRAY, [(U8, [1]), (U8, [])])), ("f", F32, 0.5), ("u", U64, 7), ("i", I32, -3)]
    out = [build(meta, [("t0", [32, 2], sc.Q8_0, blk * 2), ("t1", [64], sc.Q8_0, blk * 2)])[0]]
    q4 = g.integers(0, 256, 3 * 4 * 144, dtype=np.uint8).tobytes()
    out.append(build([("general.alignment", U32, 64)],
                     [("exps", [256, 4, 3], sc.Q4_K, q4), ("norm", [16], sc.F32, bytes(64))], align=64,
                     data_align=64)[0])
    out.append(build([("split.no", U32, 0), ("split.count", U32, 2)], [], pad=False)[0])
    out.append(build([], [("w", [32, 1, 1, 2], sc.Q8_0, blk * 2), ("bf", [8], sc.BF16, bytes(16))])[0])
    return out


@pytest.mark.skipif(shutil.which("g++") is None or not (CUDA_INC / "nvtx3").exists(), reason="needs g++ and nvtx3")
def test_mutated_files_never_read_out_of_bounds(tmp_path):
    exe = tmp_path / "gguf_fuzz"
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
           "-I", str(ROOT / "include"), "-I", str(ROOT / "strata-rs_b200" / "csrc"), "-I", str(CUDA_INC),
           str(ROOT / "strata-rs_b200" / "csrc" / "gguf.cpp"), str(ROOT / "tests" / "gguf_fuzz.cpp"), "-o", str(exe),
           "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    files = []
    for k, data in enumerate(seeds()):
        p = tmp_path / f"seed{k}.gguf"
        p.write_bytes(data)
        files.append(str(p))
    r = subprocess.run([str(exe), str(tmp_path / "fuzz.gguf"), "4000", *files], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.startswith("ok"), (r.stdout + r.stderr)[-3000:]
    opened, refused = map(int, r.stdout.split()[1:3])
    assert opened > 200 and refused > 200, r.stdout  # both outcomes were exercised
