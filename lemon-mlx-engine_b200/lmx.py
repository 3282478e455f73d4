"""ctypes binding of liblmx.so, the B200 speculative-decode library.

This is a thin host-side mirror of the C ABI in include/lmx.h.  It never
falls back to another implementation: if the CUDA library is missing or a call
fails, it raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblmx.so")

P = C.c_void_p
I = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
F = C.c_float

_lib = None


class LmxError(RuntimeError):
    pass


# Every exported symbol of include/lmx.h with (restype, argtypes).
SIGNATURES = {
    "lmx_last_error": (C.c_char_p, []),
    "lmx_version": (C.c_char_p, []),
    "lmx_device_error": (I, [C.POINTER(C.c_uint), I]),
    "lmx_quantized_matmul": (I, [P, P, P, P, P, I, I, I, I, I, P]),
    "lmx_rms_norm": (I, [P, P, P, I, I, F, P]),
    "lmx_argmax": (I, [P, I, I, P, P]),
}


def lib():
    """Load liblmx.so (raises LmxError if the CUDA extension is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LmxError(f"CUDA extension missing: {LIB_PATH} (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, what="lmx call"):
    if rc != 0:
        msg = lib().lmx_last_error().decode(errors="replace")
        raise LmxError(f"{what} failed with status {rc}: {msg}")
    return rc


def call(name, *args):
    return check(getattr(lib(), name)(*args), name)
