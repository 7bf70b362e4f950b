"""strata_cuda_gguf_moe_layer's host side on the CPU: the loader of one MoE
layer from a GGUF model (strata-core's load_layer, crates/strata-core/src/
moe.rs:147-188) is compiled with tests/gguf_layer_check.cpp, whose stand-ins
for the upload and the layer creation print what they receive. Checked: the
tensor names, the expert-range slices of the file, the geometry of every
upload, the layer description, and the errors for a missing tensor and a bad
expert range. The device side is tests/test_gguf_gpu.py."""
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import strata_cuda as sc
from gguf_writer import STRING, build
from synth import rng

ROOT = Path(__file__).resolve().parents[1]
CUDA_INC = Path("/usr/local/cuda/include")
N_EMBD, N_FF, N_FF_S, E = 256, 256, 512, 8


def layer_tensors(layer: int, g):
    q4 = lambda n_blocks: g.integers(0, 256, n_blocks * 144, dtype=np.uint8).tobytes()
    p = f"blk.{layer}."
    return [(p + "ffn_gate_inp.weight", [N_EMBD, E], sc.Q4_K, q4(E)),
            (p + "ffn_gate_exps.weight", [N_FF, N_EMBD, E], sc.Q4_K, q4(E * N_EMBD)),
            (p + "ffn_up_exps.weight", [N_FF, N_EMBD, E], sc.Q4_K, q4(E * N_EMBD)),
            (p + "ffn_down_exps.weight", [N_EMBD, N_FF, E], sc.Q4_K, q4(E * N_FF)),
            (p + "ffn_gate_shexp.weight", [N_EMBD, N_FF_S], sc.Q4_K, q4(N_FF_S)),
            (p + "ffn_up_shexp.weight", [N_EMBD, N_FF_S], sc.Q4_K, q4(N_FF_S)),
            (p + "ffn_down_shexp.weight", [N_FF_S, N_EMBD], sc.Q4_K, q4(2 * N_EMBD)),
            (p + "ffn_gate_inp_shexp.weight", [N_EMBD], sc.Q4_K, q4(1))]


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if shutil.which("g++") is None or not (CUDA_INC / "nvtx3").exists():
        pytest.skip("needs g++ and nvtx3")
    d = tmp_path_factory.mktemp("layer")
    exe = d / "gguf_layer_check"
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
           "-I", str(ROOT / "include"), "-I", str(ROOT / "strata-rs_b200" / "csrc"), "-I", str(CUDA_INC),
           str(ROOT / "strata-rs_b200" / "csrc" / "gguf.cpp"), str(ROOT / "tests" / "gguf_layer_check.cpp"),
           "-o", str(exe), "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    tensors = layer_tensors(3, rng(4321))
    data, _, _ = build([("general.architecture", STRING, "qwen35moe")], tensors)
    model = d / "moe.gguf"
    model.write_bytes(data)
    blobs = {n: b for n, _, _, b in tensors}

    def run(*args):
        r = subprocess.run([str(exe), str(model), *map(str, args)], capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, r.stdout + r.stderr
        ups = [dict(kv.split("=") for kv in ln.split()[2:]) for ln in r.stdout.splitlines() if ln.startswith("upload")]
        desc = [dict(kv.split("=") for kv in ln.split()[1:]) for ln in r.stdout.splitlines() if ln.startswith("desc")]
        rc = re.search(r"^rc (\d+) ?(.*)$", r.stdout, re.M)
        return ups, (desc[0] if desc else None), int(rc.group(1)), rc.group(2)
    return run, blobs


def test_whole_layer_with_the_shared_expert(harness):
    run, blobs = harness
    ups, desc, rc, _ = run(3, 4, 0, 0, 1)
    assert rc == 0 and len(ups) == 8
    names = [n for n, _, _, _ in layer_tensors(3, rng(0))]
    geo = [(0, E, N_EMBD), (E, N_EMBD, N_FF), (E, N_EMBD, N_FF), (E, N_FF, N_EMBD), (0, N_FF_S, N_EMBD),
           (0, N_FF_S, N_EMBD), (0, N_EMBD, N_FF_S), (0, 1, N_EMBD)]
    for u, nm, (ne, rows, cols) in zip(ups, names, geo):
        b = blobs[nm]
        assert (int(u["n_expert"]), int(u["rows"]), int(u["cols"])) == (ne, rows, cols), nm
        assert int(u["len"]) == len(b) and int(u["first"]) == b[0] and int(u["last"]) == b[-1], nm
    assert desc["handles"] == "1,2,3,4,5,6,7,8"
    assert (desc["n_embd"], desc["n_expert"], desc["top_k"], desc["n_ff"], desc["n_ff_shexp"]) == \
        (str(N_EMBD), str(E), "4", str(N_FF), str(N_FF_S))
    assert (desc["begin"], desc["end"], desc["shared"]) == ("0", str(E), "1")


def test_an_expert_parallel_rank_reads_only_its_experts(harness):
    run, blobs = harness
    ups, desc, rc, _ = run(3, 2, 2, 6, 0)
    assert rc == 0 and len(ups) == 4  # router + the three expert tensors; no shared expert here
    per = {1: N_EMBD * 144, 2: N_EMBD * 144, 3: N_FF * 144}
    names = [n for n, _, _, _ in layer_tensors(3, rng(0))]
    for i in (1, 2, 3):
        b, u = blobs[names[i]], ups[i]
        part = b[2 * per[i]:6 * per[i]]
        assert int(u["n_expert"]) == 4 and int(u["len"]) == len(part)
        assert int(u["first"]) == part[0] and int(u["last"]) == part[-1]
    assert desc["handles"] == "1,2,3,4,0,0,0,0" and (desc["begin"], desc["end"], desc["shared"]) == ("2", "6", "0")
    assert desc["n_expert"] == str(E)  # ids stay global


def test_missing_tensor_and_bad_range(harness):
    run, _ = harness
    ups, desc, rc, msg = run(4, 4, 0, 0, 1)
    assert rc == sc.ERR_TENSOR_NOT_FOUND and "blk.4.ffn_gate_inp.weight" in msg and not ups and desc is None
    ups, desc, rc, msg = run(3, 4, 6, 9, 1)
    assert rc == sc.ERR_INVALID and "[6, 9)" in msg and not ups
