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
