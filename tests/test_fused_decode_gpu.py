"""The fused small-batch decode forward (decode.cuh): the whole decoder stack
for at most 16 token rows in one persistent kernel, in tensor-core mode.

Checked against the oracle taking the same numerical form per block (its
tensor-core emulation: dequantize-then-dot for blocks of >= 16 rows, the
canonical order below) on Qwen3-0.6B layer widths (hidden 1024, 16 q / 8 kv
heads, FFN 3072) with draft-like blocks (T = 2 and T = 1 per sequence, as
the speculative loop's draft forwards) and verify-like blocks (T = 5), with
rollbacks between them; plus run-to-run determinism and the switch that
turns the path off."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

CFG = dict(hidden=1024, layers=3, inter=3072, heads=16, kv_heads=8, head_dim=128, vocab=2048,
           rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)


def oracle_cfg(cfg):
    d = dict(cfg)
    d["group"] = d.pop("group_size")
    return O.ModelCfg(**d)


def within(got, ref, what, kv_bits):
    # 3 layers of Qwen3-0.6B widths after a prefill whose 40-row chunks take
    # the tcgen05 path: the accumulation-order drift against the oracle's
    # emulation reaches ~0.03 (measured), so the bound is 4e-2 + ulp
    g, r = O.bf16_to_f32(got), O.bf16_to_f32(ref)
    diff = np.abs(g - r)
    lim = 4e-2 + np.abs(r) * 2.0 ** -7
    if kv_bits != 16:
        # a quantized cache code can flip on a one-ulp K/V difference and move
        # every logit of the rows that read it (see test_engine_gpu): bounded
        # by 1e-1 per logit
        assert not (diff > 1e-1 + lim).any(), f"{what}: max |diff| {diff.max():.4g}"
        return
    assert not (diff > lim).any(), f"{what}: {int((diff > lim).sum())} beyond 4e-2 + ulp, max {diff.max():.4g}"


@pytest.fixture(autouse=True)
def fused_off_after(lmx):
    yield
    lmx.call("lmx_set_fused_decode", 0)


@pytest.fixture(scope="module")
def models(lmx, cuda):
    out = {}
    for bits in (4, 8):
        cfg = dict(CFG, bits=bits, tied=1 if bits == 4 else 0)
        out[bits] = (cfg, lmx.Model(cfg, 4321 + bits),
                     O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), 4321 + bits))
    yield out
    for cfg, g, o in out.values():
        g.close()
        O.lib().orc_model_free(o)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("kv_bits", [16, 8, 4])
@pytest.mark.parametrize("B", [1, 3, 8])
def test_fused_decode_blocks_match_oracle(lmx, models, mma_threshold, bits, kv_bits, B):
    cfg, g, o = models[bits]
    L, V = cfg["layers"], cfg["vocab"]
    lmx.call("lmx_set_fused_decode", 1)
    mma_threshold(16)
    gc = C.c_void_p()
    cap = 400
    lmx.call("lmx_cache_create", g.h, L, B, cap, kv_bits, 40, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, cap, kv_bits)
    rng = np.random.RandomState(B * 100 + kv_bits + bits)
    # prefill crossing a 128-key split boundary, then draft / verify blocks;
    # R = B*T <= 16 takes the fused kernel
    blocks = [130, 2, 1, 1, 5, 1, 2, 5]
    try:
        for i, T in enumerate(blocks):
            if i == 0:
                # prefill in chunks of <= 40 rows per sequence
                for t0 in range(0, T, 40):
                    tn = min(40, T - t0)
                    tok = rng.randint(0, V, (B, tn)).astype(np.int32)
                    lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, tn, None)
                    assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, tn, None) == 0
                continue
            if i == 5:  # roll sequences back by different amounts (speculative rejection)
                for b in range(B):
                    n = C.c_int()
                    lmx.call("lmx_cache_len", gc, b, C.byref(n))
                    pos = n.value - 1 - (b % 3)
                    lmx.call("lmx_cache_set_position", gc, b, pos)
                    O.lib().orc_cache_set_position(oc, b, pos)
            tok = rng.randint(0, V, (B, T)).astype(np.int32)
            gl = np.zeros((B, T, V), np.uint16)
            ol = np.zeros((B, T, V), np.uint16)
            lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
            assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
            within(gl, ol, f"block {i} (B={B}, T={T})", kv_bits)
            for b in range(B):
                n = C.c_int()
                lmx.call("lmx_cache_len", gc, b, C.byref(n))
                assert n.value == O.lib().orc_cache_len(oc, b)
        code = C.c_uint(0)
        lmx.call("lmx_device_error", C.byref(code), 1)
        assert code.value == 0, hex(code.value)
    finally:
        lmx.call("lmx_cache_free", gc)
        O.lib().orc_cache_free(oc)


def test_fused_decode_deterministic_and_switchable(lmx, models, mma_threshold):
    cfg, g, o = models[4]
    L, V, B = cfg["layers"], cfg["vocab"], 8
    mma_threshold(16)
    rng = np.random.RandomState(11)
    pre = rng.randint(0, V, (B, 20)).astype(np.int32)
    blk = rng.randint(0, V, (B, 1)).astype(np.int32)
    outs = []
    for fused in (1, 1, 0):
        lmx.call("lmx_set_fused_decode", fused)
        gc = C.c_void_p()
        lmx.call("lmx_cache_create", g.h, L, B, 64, 4, 20, C.byref(gc))
        lmx.call("lmx_forward", g.h, gc, L, pre.ctypes.data, B, 20, None)
        gl = np.zeros((B, 1, V), np.uint16)
        lmx.call("lmx_forward", g.h, gc, L, blk.ctypes.data, B, 1, gl.ctypes.data)
        lmx.call("lmx_cache_free", gc)
        outs.append(gl)
    np.testing.assert_array_equal(outs[0], outs[1])  # deterministic
    # the per-op path (small-batch tensor-core GEMV) agrees within tolerance
    within(outs[0], outs[2], "fused vs per-op", 4)
    assert lmx.lib().lmx_set_fused_decode(2) != 0
