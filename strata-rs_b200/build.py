"""Builds libstrata_cuda.so in-tree with nvcc for sm_100a.

Every .cu (and host-only .cpp) under csrc/ is compiled to an object with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`, then linked into one
shared library next to this file. Objects go to _build/ (git-ignored).
Run: python strata-rs_b200/build.py [--verbose-ptxas]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
OUT = HERE / "libstrata_cuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-Wall", "--expt-relaxed-constexpr",
            "-I", str(HERE.parent / "include"), "-I", str(CSRC)]


def _needs(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((HERE.parent / "include").glob("*.h"))
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: Path, ptxas_v: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if not _needs(obj, src):
        return obj, ""
    cmd = [NVCC, *ARCH, *CXXFLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(ptxas_v: bool = False, quiet: bool = True) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_v), srcs))
    objs = [o for o, _ in results]
    if not quiet or ptxas_v:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    if not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(OUT), *map(str, objs),
               "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(ptxas_v="--verbose-ptxas" in sys.argv, quiet=False))
