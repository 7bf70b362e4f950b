"""The host-side copy code of strata-rs_b200/csrc/staging.h on the CPU: the
chunk and piece arithmetic that strata_cuda_upload / strata_cuda_upload_many
run before any copy reaches the device, and the threaded host copy of large
results, compiled into a host program with address and undefined-behaviour
checks (then with the thread checker) and run over random sizes."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_staging_plan_moves_every_byte_once(tmp_path):
    exe = tmp_path / "staging_check"
    for san in ("address,undefined", "thread"):  # bounds and UB; then races of the threaded copy
        cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", f"-fsanitize={san}", "-fno-sanitize-recover=all",
               "-pthread", "-I", str(ROOT / "strata-rs_b200" / "csrc"), str(ROOT / "tests" / "staging_check.cpp"),
               "-o", str(exe)]
        subprocess.run(cmd, check=True, capture_output=True, text=True)
        r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and r.stdout.strip() == "ok", (san, r.stdout + r.stderr)
