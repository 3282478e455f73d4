"""The C-ABI library loads and exports every symbol include/lmx.h declares."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "lmx.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lmx_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(lmx):
    L = lmx.lib()
    syms = declared_symbols()
    assert len(syms) >= 5
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(syms) <= set(lmx.SIGNATURES), set(syms) - set(lmx.SIGNATURES)


def test_version_and_error_text(lmx):
    L = lmx.lib()
    assert L.lmx_version().startswith(b"lmx-b200")
    # an invalid call fails with a status, not an exception or a crash
    rc = L.lmx_quantized_matmul(None, None, None, None, None, 1, 8, 64, 32, 4, None)
    assert rc == 2 and b"group_size" in L.lmx_last_error()


def test_tensor_core_thresholds_host_side(lmx):
    # the process-wide path switches are host state: settable and validated
    # without a GPU; restored to their defaults afterwards
    L = lmx.lib()
    assert L.lmx_mma_min_m() == 16 and L.lmx_gemv_tc_min_m() == 4
    try:
        assert L.lmx_set_gemv_tc_min_m(17) != 0 and b"gemv_tc_min_m" in L.lmx_last_error()
        assert L.lmx_set_gemv_tc_min_m(-1) != 0
        assert L.lmx_set_gemv_tc_min_m(0) == 0 and L.lmx_gemv_tc_min_m() == 0
        assert L.lmx_set_gemv_tc_min_m(8) == 0 and L.lmx_gemv_tc_min_m() == 8
        assert L.lmx_set_mma_min_m(0) == 0 and L.lmx_mma_min_m() == 0
    finally:
        L.lmx_set_gemv_tc_min_m(4)
        L.lmx_set_mma_min_m(16)
