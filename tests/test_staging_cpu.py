"""The upload staging plan (strata-rs_b200/csrc/staging.h) on the CPU: the
chunk and piece arithmetic that strata_cuda_upload / strata_cuda_upload_many
run before any copy reaches the device, compiled into a host program with
address and undefined-behaviour checks and run over random range lists."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_staging_plan_moves_every_byte_once(tmp_path):
    exe = tmp_path / "staging_check"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=all", "-I", str(ROOT / "strata-rs_b200" / "csrc"),
           str(ROOT / "tests" / "staging_check.cpp"), "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
