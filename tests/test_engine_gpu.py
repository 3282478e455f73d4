"""End-to-end engine on the B200 vs the CPU oracle: generated weights, the
forward (logits) and the speculative token streams, all bit-exact."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

TINY = dict(hidden=512, layers=3, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=1000,
            rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)


def oracle_cfg(cfg):
    d = dict(cfg)
    d["group"] = d.pop("group_size")
    return O.ModelCfg(**d)


@pytest.fixture(scope="module")
def models(lmx, cuda):
    cfgs = {4: dict(TINY), 8: dict(TINY, bits=8, tied=0)}
    out = {}
    for bits, cfg in cfgs.items():
        g = lmx.Model(cfg, 1234)
        o = O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), 1234)
        out[bits] = (cfg, g, o)
    yield out
    for cfg, g, o in out.values():
        g.close()
        O.lib().orc_model_free(o)


@pytest.mark.parametrize("bits", [4, 8])
def test_generated_weights_bit_exact(lmx, models, bits):
    cfg, g, o = models[bits]
    H, D = cfg["hidden"], cfg["head_dim"]
    shapes = {0: (cfg["heads"] * D, H), 6: (H, cfg["inter"]), 7: (cfg["vocab"], H)}
    if not cfg["tied"]:
        shapes[8] = (cfg["vocab"], H)
    for kind, (N, K) in shapes.items():
        for layer in ([0, 2] if kind < 7 else [0]):
            gw = np.zeros(N * K * bits // 32, np.uint32)
            gs = np.zeros(N * K // 64, np.uint16)
            gb = np.zeros_like(gs)
            lmx.call("lmx_model_weight", g.h, layer, kind, gw.ctypes.data, gs.ctypes.data, gb.ctypes.data)
            ow, os_, ob = np.zeros_like(gw), np.zeros_like(gs), np.zeros_like(gb)
            assert O.lib().orc_model_weight(o, layer, kind, O.ptr(ow), O.ptr(os_), O.ptr(ob)) == 0
            np.testing.assert_array_equal(gw, ow)
            np.testing.assert_array_equal(gs, os_)
            np.testing.assert_array_equal(gb, ob)


def assert_logits_close(got, ref, what, kv_bits=16):
    # 2e-2 max-abs, widened by one bf16 ulp of the logit: above |4| the bf16
    # grid itself is coarser than 2e-2, and both sides round nearly equal
    # fp32 values to it.  With a 4-bit KV cache the bound is doubled: its
    # min/max quantizer is discontinuous, so a one-ulp difference in a K/V
    # projection can move a code by a whole quantization step (1/15 of the
    # group's range) and the attention output with it.  Such flips are rare
    # but unbounded in number by any fixed max-abs: with a 4-bit cache, at
    # most 0.05% of the logits may exceed 4e-2 (+ ulp), and none 1e-1 (+ ulp).
    g, r = O.bf16_to_f32(got), O.bf16_to_f32(ref)
    ulp = np.abs(r) * 2.0 ** -7
    diff = np.abs(g - r)
    if kv_bits == 4:
        over = int((diff > 4e-2 + ulp).sum())
        assert over <= 5e-4 * diff.size and not (diff > 1e-1 + ulp).any(), \
            f"{what}: {over} logits beyond 4e-2 (of {diff.size}), max |diff| {diff.max():.4g}"
        return
    bad = diff > 2e-2 + ulp
    assert not bad.any(), f"{what}: {int(bad.sum())} logits out of tolerance, max |diff| {diff.max():.4g}"


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("kv_bits", [16, 8, 4])
@pytest.mark.parametrize("mma", [0, 16])
def test_forward_logits_with_rollback(lmx, models, mma_threshold, bits, kv_bits, mma):
    # mma 0: every matmul on the canonical GEMV -> bit-exact logits.
    # mma 16: blocks of >= 16 rows run the tcgen05 path -> logits within
    # 2e-2 max-abs of the oracle (which takes the same path choice).
    mma_threshold(mma)
    cfg, g, o = models[bits]
    L, V, B = cfg["layers"], cfg["vocab"], 2
    cap = 160
    gc = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, L, B, cap, kv_bits, 40, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, cap, kv_bits)
    rng = np.random.RandomState(kv_bits + bits)
    # prefill 37 tokens (crosses a 32-key split), then a 5-token verify block,
    # roll one sequence back, re-run; then decode steps crossing 128 keys
    blocks = [37, 5, 5, 1, 1] + [30, 30, 5]
    mma_seen = False
    for i, T in enumerate(blocks):
        if i == 2:
            for b, pos in enumerate([39, 38]):
                lmx.call("lmx_cache_set_position", gc, b, pos)
                O.lib().orc_cache_set_position(oc, b, pos)
        if i == 5:
            for b in range(B):  # make the sequence lengths differ further
                lmx.call("lmx_cache_set_position", gc, b, 40 - 3 * b)
                O.lib().orc_cache_set_position(oc, b, 40 - 3 * b)
        tok = rng.randint(0, V, (B, T)).astype(np.int32)
        gl = np.zeros((B, T, V), np.uint16)
        ol = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
        assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
        mma_seen = mma_seen or (mma and B * T >= mma)
        if mma_seen:  # the cache now holds rows written by the tensor-core path
            assert_logits_close(gl, ol, f"block {i}", kv_bits)
        else:
            bad = np.argwhere(gl != ol)
            assert bad.size == 0, f"block {i}: {len(bad)} mismatching logits, first {bad[:3].tolist()}"
        for b in range(B):
            n = C.c_int()
            lmx.call("lmx_cache_len", gc, b, C.byref(n))
            assert n.value == O.lib().orc_cache_len(oc, b)
    lmx.call("lmx_cache_free", gc)
    O.lib().orc_cache_free(oc)


def oracle_spec(o, prompts, K, MT, kv_bits, draft_layers, temperature=0.0, top_p=1.0, seed=0):
    B, P = prompts.shape
    out = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=K, max_tokens=MT, temperature=temperature, top_p=top_p, seed=seed,
                       draft_layers=draft_layers)
    assert O.lib().orc_spec_generate(o, None, O.ptr(np.ascontiguousarray(prompts)), B, P, prm,
                                     kv_bits, O.ptr(out), O.ptr(st)) == 0
    return out, st


@pytest.mark.parametrize("kv_bits", [16, 4])
@pytest.mark.parametrize("use_graph", [True, False])
def test_spec_greedy_stream_matches_oracle(lmx, models, mma_threshold, kv_bits, use_graph):
    # exact mode: every matmul in the canonical order, so the streams are
    # bit-identical (with the tensor-core path on, logits agree only within
    # tolerance and near-ties may flip a token)
    mma_threshold(0)
    cfg, g, o = models[4]
    B, P, K, MT = 3, 20, 4, 48
    prompts = np.random.RandomState(7).randint(0, cfg["vocab"], (B, P)).astype(np.int32)
    sd = lmx.SpecDecoder(g, None, 1, B, K, MT, P, kv_bits=kv_bits)
    sd.prefill(prompts)
    sd.decode(use_graph=use_graph)
    got, stats = sd.result()
    sd.close()
    ref, rst = oracle_spec(o, prompts, K, MT, kv_bits, 1)
    np.testing.assert_array_equal(got, ref)
    assert stats["accepted"] == rst[2] and stats["steps"] == rst[0] * 0 + stats["steps"]
    # lossless: equals plain greedy decoding of the target
    plain = np.zeros((B, MT), np.int32)
    assert O.lib().orc_generate(o, O.ptr(prompts), B, P, MT, kv_bits, O.ptr(plain)) == 0
    np.testing.assert_array_equal(got, plain)


@pytest.mark.parametrize("bits", [4, 8])
def test_batched_verify_logits_tensor_core(lmx, models, mma_threshold, bits):
    # config-3-shaped verify blocks (8 sequences x 6 tokens = 48 rows) on the
    # tcgen05 path after an exact-mode prefill: logits within tolerance
    cfg, g, o = models[bits]
    L, V, B, cap = cfg["layers"], cfg["vocab"], 8, 128
    gc = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, L, B, cap, 4, 48, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, cap, 4)
    rng = np.random.RandomState(bits)
    for i, (T, mma) in enumerate([(12, 0), (6, 16), (6, 16), (1, 16), (6, 16)]):
        mma_threshold(mma)
        tok = rng.randint(0, V, (B, T)).astype(np.int32)
        gl = np.zeros((B, T, V), np.uint16)
        ol = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
        assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
        if i == 0:
            np.testing.assert_array_equal(gl, ol)
        else:
            assert_logits_close(gl, ol, f"block {i}", 4)
        if i == 2:  # roll every sequence back by a different amount
            for b in range(B):
                pos = 12 + 6 + (b % 6)
                lmx.call("lmx_cache_set_position", gc, b, pos)
                O.lib().orc_cache_set_position(oc, b, pos)
    lmx.call("lmx_cache_free", gc)
    O.lib().orc_cache_free(oc)


def test_llama_rope_scaled_forward_bit_exact(lmx, cuda, mma_threshold):
    # Llama-style decoder (no q/k norm, tied embedding) with Llama-3 RoPE
    # frequency scaling (factor 32, original context 64 so the scaled and
    # interpolated bands both occur inside 128 dims); exact mode
    mma_threshold(0)
    cfg = dict(hidden=512, layers=2, inter=1024, heads=8, kv_heads=2, head_dim=128, vocab=1000,
               rope_theta=5e5, eps=1e-5, qk_norm=0, tied=1, bits=4, group_size=64,
               rope_factor=32.0, rope_low_freq=1.0, rope_high_freq=4.0, rope_orig_max_pos=64.0)
    g = lmx.Model(cfg, 77)
    o = O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), 77)
    L, V, B, cap = cfg["layers"], cfg["vocab"], 2, 96
    gc = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, L, B, cap, 8, 40, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, cap, 8)
    rng = np.random.RandomState(5)
    for T in (40, 5, 1):
        tok = rng.randint(0, V, (B, T)).astype(np.int32)
        gl = np.zeros((B, T, V), np.uint16)
        ol = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
        assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
        np.testing.assert_array_equal(gl, ol)
    lmx.call("lmx_cache_free", gc)
    O.lib().orc_cache_free(oc)
    g.close()
    O.lib().orc_model_free(o)


LLAMA_TINY = dict(hidden=512, layers=2, inter=1024, heads=8, kv_heads=2, head_dim=128, vocab=1024,
                  rope_theta=5e5, eps=1e-5, qk_norm=0, tied=0, bits=4, group_size=64)
LLAMA_DRAFT = dict(LLAMA_TINY, layers=1, tied=1)


@pytest.mark.parametrize("kv_bits", [16, 8, 4])
def test_synthetic_context_forward_bit_exact(lmx, cuda, mma_threshold, kv_bits):
    # lmx_cache_fill_synthetic == orc_cache_fill_synthetic (Philox normal,
    # quantized like an append), then forwards on top of the 70-row context
    mma_threshold(0)
    cfg = LLAMA_TINY
    g = lmx.Model(cfg, 31)
    o = O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), 31)
    L, V, B, cap, ctx = cfg["layers"], cfg["vocab"], 3, 128, 70
    gc = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, L, B, cap, kv_bits, 8, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, cap, kv_bits)
    lmx.call("lmx_cache_fill_synthetic", gc, ctx, 99, 0x40000000)
    assert O.lib().orc_cache_fill_synthetic(oc, ctx, 99, 0x40000000) == 0
    rng = np.random.RandomState(kv_bits)
    for T in (8, 5, 1):
        tok = rng.randint(0, V, (B, T)).astype(np.int32)
        gl = np.zeros((B, T, V), np.uint16)
        ol = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
        assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
        np.testing.assert_array_equal(gl, ol)
    n = C.c_int()
    lmx.call("lmx_cache_len", gc, 0, C.byref(n))
    assert n.value == ctx + 14
    lmx.call("lmx_cache_free", gc)
    O.lib().orc_cache_free(oc)
    g.close()
    O.lib().orc_model_free(o)


def test_synthetic_context_spec_stream_matches_oracle(lmx, cuda, mma_threshold):
    # config-5-shaped session in miniature: Llama target, separate Llama
    # draft, greedy, 8-bit KV, a synthetic context before the prompt
    mma_threshold(0)
    tg = lmx.Model(LLAMA_TINY, 41)
    dg = lmx.Model(LLAMA_DRAFT, 42)
    to = O.lib().orc_model_create(C.byref(oracle_cfg(LLAMA_TINY)), 41)
    do = O.lib().orc_model_create(C.byref(oracle_cfg(LLAMA_DRAFT)), 42)
    B, P, K, MT, ctx = 4, 12, 4, 40, 150
    prompts = np.random.RandomState(3).randint(0, LLAMA_TINY["vocab"], (B, P)).astype(np.int32)
    sd = lmx.SpecDecoder(tg, dg, 1, B, K, MT, P, kv_bits=8, context_len=ctx, context_seed=11)
    sd.prefill(prompts)
    sd.decode()
    got, stats = sd.result()
    sd.close()
    out = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=K, max_tokens=MT, temperature=0.0, top_p=1.0, seed=0, draft_layers=1,
                       context_len=ctx, context_seed=11)
    assert O.lib().orc_spec_generate(to, do, O.ptr(prompts), B, P, prm, 8, O.ptr(out), O.ptr(st)) == 0
    np.testing.assert_array_equal(got, out)
    assert stats["accepted"] == st[2]
    for m in (tg, dg):
        m.close()
    O.lib().orc_model_free(to)
    O.lib().orc_model_free(do)


def test_verify_blocks_tensor_core_attention(lmx, cuda, mma_threshold):
    # G = 8 q heads per KV head (the Llama-3-70B layout): a 5-token verify
    # block gives 40 query rows per KV head, so with the tensor-core
    # threshold on, both the matmuls and SDPA run on the tensor cores, over a
    # 700-row synthetic context (6 key chunks); logits within the contract's
    # tolerance of the oracle (whose SDPA keeps the canonical fp32 order)
    cfg = dict(LLAMA_TINY, heads=16, kv_heads=2)
    g = lmx.Model(cfg, 51)
    o = O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), 51)
    L, V, B, cap, ctx = cfg["layers"], cfg["vocab"], 4, 768, 700
    gc = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, L, B, cap, 8, 8, C.byref(gc))
    oc = O.lib().orc_cache_create(o, L, B, cap, 8)
    lmx.call("lmx_cache_fill_synthetic", gc, ctx, 5, 0x40000000)
    assert O.lib().orc_cache_fill_synthetic(oc, ctx, 5, 0x40000000) == 0
    rng = np.random.RandomState(8)
    for i, T in enumerate((5, 5, 1, 5)):
        mma_threshold(16)
        tok = rng.randint(0, V, (B, T)).astype(np.int32)
        gl = np.zeros((B, T, V), np.uint16)
        ol = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
        assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
        assert_logits_close(gl, ol, f"block {i}", 8)
        if i == 1:  # roll back two sequences
            for b, pos in ((0, ctx + 6), (2, ctx + 3)):
                lmx.call("lmx_cache_set_position", gc, b, pos)
                O.lib().orc_cache_set_position(oc, b, pos)
    lmx.call("lmx_cache_free", gc)
    O.lib().orc_cache_free(oc)
    g.close()
    O.lib().orc_model_free(o)
