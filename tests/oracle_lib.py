"""ctypes binding of the CPU oracle (oracle/liboracle.so) -- test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module; the product path never does.
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
LIB_PATH = os.path.join(ORACLE_DIR, "liboracle.so")

_lib = None


def build():
    subprocess.check_call(["make", "-s", "-C", ORACLE_DIR])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
U32 = C.c_uint32
F = C.c_float


class ModelCfg(C.Structure):
    _fields_ = [("hidden", I), ("layers", I), ("inter", I), ("heads", I), ("kv_heads", I),
                ("head_dim", I), ("vocab", I), ("rope_theta", F), ("eps", F), ("qk_norm", I),
                ("tied", I), ("bits", I), ("group", I), ("rope_factor", F), ("rope_low_freq", F),
                ("rope_high_freq", F), ("rope_orig_max_pos", F)]


class HybridCfg(C.Structure):
    _fields_ = [("hidden", I), ("layers", I), ("attn_every", I), ("heads", I), ("kv_heads", I),
                ("lin_k_heads", I), ("lin_v_heads", I), ("experts", I), ("top_k", I), ("expert_inter", I),
                ("shared_inter", I), ("vocab", I), ("rope_theta", F), ("eps", F), ("bits", I)]


class SpecParams(C.Structure):
    _fields_ = [("K", I), ("max_tokens", I), ("temperature", F), ("top_p", F), ("seed", U64),
                ("draft_layers", I), ("context_len", I), ("context_seed", U64)]


def _declare(L):
    sig = {
        "orc_exp": (F, [F]),
        "orc_f32_to_bf16": (C.c_uint16, [F]),
        "orc_bf16_to_f32": (F, [C.c_uint16]),
        "orc_philox": (None, [U64, P, P]),
        "orc_gen_normal_bf16": (None, [U64, U32, F, I64, P]),
        "orc_normal_scale": (F, [F]),
        "orc_gen_words": (None, [U64, U32, I64, P]),
        "orc_gen_tokens": (None, [U64, U32, I64, I, P]),
        "orc_uniform24": (U32, [U64, U32, U32, U32, U32]),
        "orc_quantize": (I, [P, I, I, I, I, P, P, P]),
        "orc_dequantize": (I, [P, P, P, I, I, I, I, P]),
        "orc_gen_sweep_weights": (I, [U64, U32, I, I, I, P, P, P]),
        "orc_qmm": (I, [P, P, P, P, P, I, I, I, I, I]),
        "orc_set_mma_min_m": (None, [I]),
        "orc_mma_min_m": (I, []),
        "orc_set_tcs_max_m": (None, [I]),
        "orc_tcs_max_m": (I, []),
        "orc_rms_norm": (None, [P, P, P, I, I, F]),
        "orc_rope_table": (None, [I, I, F, P, P]),
        "orc_rope_table_scaled": (None, [I, I, F, F, F, F, F, P, P]),
        "orc_rope": (None, [P, P, I, I, I, P, P]),
        "orc_swiglu": (None, [P, P, P, I64]),
        "orc_add": (None, [P, P, P, I64]),
        "orc_argmax": (None, [P, I, I, P]),
        "orc_sdpa": (None, [P, P, P, P, I, I, I, I, I, I, F]),
        "orc_sample": (I, [P, I, F, F, U32]),
        "orc_accept_greedy": (I, [P, P, I, I, P]),
        "orc_accept_stochastic": (I, [P, P, P, I, I, F, F, P, U32, P]),
        "orc_model_create": (P, [C.POINTER(ModelCfg), U64]),
        "orc_model_free": (None, [P]),
        "orc_model_weight": (I, [P, I, I, P, P, P]),
        "orc_model_set_weight": (I, [P, I, I, I, P, P, P]),
        "orc_model_set_norm": (I, [P, I, I, P]),
        "orc_cache_create": (P, [P, I, I, I, I]),
        "orc_cache_fill_synthetic": (I, [P, I, U64, U32]),
        "orc_model_set_tp": (I, [P, I]),
        "orc_log": (F, [F]),
        "orc_hybrid_create": (P, [C.POINTER(HybridCfg), U64]),
        "orc_hybrid_free": (None, [P]),
        "orc_hybrid_state_create": (P, [P, I, I, I]),
        "orc_hybrid_state_free": (None, [P]),
        "orc_hybrid_forward": (I, [P, P, P, I, I, P]),
        "orc_hybrid_spec_generate": (I, [P, P, I, I, I, I, P, P]),
        "orc_gdn_verify": (I, [I, I, I, I, P, P, P, P, P, P, P, P, F, P, P, P, P]),
        "orc_gdn_commit": (I, [I, I, I, I, P, P, P, P, P]),
        "orc_moe_route": (I, [P, I, I, I, P, P]),
        "orc_moe_experts": (I, [P, I, I, I, I, I, P, P, P, P, P, P, P, P, P, P, P, I, P]),
        "orc_cache_free": (None, [P]),
        "orc_cache_len": (I, [P, I]),
        "orc_cache_set_position": (None, [P, I, I]),
        "orc_forward": (I, [P, P, I, P, I, I, P]),
        "orc_spec_generate": (I, [P, P, P, I, I, C.POINTER(SpecParams), I, P, P]),
        "orc_generate": (I, [P, P, I, I, I, I, P]),
        "orc_threads": (I, []),
        "orc_set_threads": (I, [I]),
        "orc_set_gdn_state_bf16": (None, [I]),
        "orc_set_kv_quirk": (None, [I]),
        "orc_kv_quirk_alloc": (I, [I]),
        "orc_spec_session": (P, [P, P, P, I, I, C.POINTER(SpecParams), I]),
        "orc_spec_session_step": (I, [P, I]),
        "orc_spec_session_result": (None, [P, P, P]),
        "orc_spec_session_free": (None, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


# ---- bf16 helpers (numpy, uint16 bit patterns) ----
def bf16_to_f32(u16):
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f):
    u = np.asarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


# ---- thin numpy-facing wrappers ----
def gen_normal_bf16(seed, tid, std, n):
    out = np.empty(n, np.uint16)
    lib().orc_gen_normal_bf16(seed, tid, std, n, ptr(out))
    return out


def gen_sweep_weights(seed, tid, N, K, bits):
    wq = np.empty((N, K * bits // 32), np.uint32)
    s = np.empty((N, K // 64), np.uint16)
    b = np.empty((N, K // 64), np.uint16)
    assert lib().orc_gen_sweep_weights(seed, tid, N, K, bits, ptr(wq), ptr(s), ptr(b)) == 0
    return wq, s, b


def quantize(w_bf16, group, bits):
    N, K = w_bf16.shape
    wq = np.empty((N, K * bits // 32), np.uint32)
    s = np.empty((N, K // group), np.uint16)
    b = np.empty((N, K // group), np.uint16)
    assert lib().orc_quantize(ptr(np.ascontiguousarray(w_bf16)), N, K, group, bits, ptr(wq),
                              ptr(s), ptr(b)) == 0
    return wq, s, b


def dequantize(wq, s, b, K, group, bits):
    N = wq.shape[0]
    out = np.empty((N, K), np.uint16)
    assert lib().orc_dequantize(ptr(wq), ptr(s), ptr(b), N, K, group, bits, ptr(out)) == 0
    return out


def qmm(x_bf16, wq, s, b, bits, group=64):
    M, K = x_bf16.shape
    N = wq.shape[0]
    y = np.empty((M, N), np.uint16)
    rc = lib().orc_qmm(ptr(np.ascontiguousarray(x_bf16)), ptr(wq), ptr(s), ptr(b), ptr(y), M, N,
                       K, group, bits)
    assert rc == 0
    return y


def rms_norm(x_bf16, w_bf16, eps):
    rows, dim = x_bf16.shape
    y = np.empty_like(x_bf16)
    lib().orc_rms_norm(ptr(np.ascontiguousarray(x_bf16)), ptr(w_bf16), ptr(y), rows, dim, eps)
    return y


def argmax(logits_bf16):
    rows, V = logits_bf16.shape
    out = np.empty(rows, np.int32)
    lib().orc_argmax(ptr(np.ascontiguousarray(logits_bf16)), rows, V, ptr(out))
    return out


def uniform24(seed, seq, step, slot, stream):
    return lib().orc_uniform24(seed, seq, step, slot, stream)


QWEN3_06B = dict(hidden=1024, layers=28, inter=3072, heads=16, kv_heads=8, head_dim=128,
                 vocab=151936, rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group=64)
