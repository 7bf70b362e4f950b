"""The C ABI library builds, loads without a GPU, and exports every entry
point include/strata_cuda.h declares (no compute calls here)."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

import strata_cuda as sc

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(strata_cuda_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def libso():
    if not sc.LIB_PATH.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("strata_build", ROOT / "strata-rs_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return sc.lib()


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ["strata_cuda_create", "strata_cuda_upload", "strata_cuda_gemv", "strata_cuda_expert_gemv",
                 "strata_cuda_dequant", "strata_cuda_last_error"]:
        assert must in names


def test_every_declared_symbol_is_exported(libso):
    out = subprocess.run(["nm", "-D", "--defined-only", str(sc.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(strata_cuda_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for n in declared_functions():
        assert hasattr(libso, n)


def test_name_and_version(libso):
    assert libso.strata_cuda_name() == b"cuda"
    assert libso.strata_cuda_abi_version() == 1


def test_null_handles_are_rejected(libso):
    assert libso.strata_cuda_destroy(None) == sc.ERR_INVALID
    assert libso.strata_cuda_free_weight(None) == sc.ERR_INVALID
    assert libso.strata_cuda_gemv(None, None, None, None, 1) == sc.ERR_INVALID
    assert libso.strata_cuda_create(0, None) == sc.ERR_INVALID


def test_no_device_reports_an_error_instead_of_crashing(libso):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = C.c_void_p()
    assert libso.strata_cuda_create(0, C.byref(h)) != sc.OK
    assert not h.value
