"""CPU checks of the C-ABI library: it builds, loads, and exports every symbol
``include/isp_b200.h`` declares (no compute calls without a GPU)."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"^\s*(?:int|const char \*)\s*(isp_\w+)\s*\(", text, flags=re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    from inspark_proper_format_b200 import _lib, build
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"isp_norm_quant", "isp_fir_snake", "isp_scaled_gemm", "isp_gated_up"} <= names


def test_library_exports_every_declared_symbol(lib):
    from inspark_proper_format_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\b(isp_\w+)\b", out))
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert declared_symbols() == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_status_strings_and_version(lib):
    assert lib.isp_version() >= 100
    assert lib.isp_status_string(0) == b"ok"
    assert b"sm_100" in lib.isp_status_string(4)


def test_library_is_sm100a_only():
    from inspark_proper_format_b200 import build
    assert "arch=compute_100a,code=sm_100a" in build.ARCH_FLAGS


def test_host_validation_runs_before_any_device_work(lib):
    # NULL input / bad dtype are rejected on the host, without touching a GPU.
    assert lib.isp_norm_quant(None, 0, 4, 512, None, None, 1e-6, 1.0, 0, 0, 1.0, None, None, None, None) == 7
    assert lib.isp_fir_snake(None, 1, 1, 4, None, None, None, None, None, 1, None, 1.0, None) == 7
    # limits outside 1 us .. 100 ms are refused before any device access
    assert lib.isp_wait_selftest(10, None) == 7
    assert lib.isp_wait_selftest(10**9, None) == 7
    assert lib.isp_int8_nonlinear_value(None, None, 4, 384, 512, 1, 0.01, None, None, None, None, None) == 7
