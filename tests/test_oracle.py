"""CPU oracle pinned against the reference's own golden vectors and tests."""
import math
import os

import numpy as np
import pytest

import oracle_lib as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def f32(u16):
    return O.bf16_to_f32(u16)


@pytest.mark.parametrize("bits", [4, 8])
def test_packing_order_matches_reference(bits):
    # debug_numerical_trace.py:67-100 / debug_layer0_reference.py:53-82 with
    # scale 1, bias 0 return the raw codes: LSB-first packing, exact.
    w = GOLD[f"q{bits}_w"]
    N, K = w.shape[0], w.shape[1] * 32 // bits
    ones = np.full((N, K // 64), O.f32_to_bf16(np.float32(1.0)), np.uint16)
    zeros = np.zeros((N, K // 64), np.uint16)
    codes = f32(O.dequantize(w, ones, zeros, K, 64, bits))
    np.testing.assert_array_equal(codes, GOLD[f"q{bits}_codes"])


@pytest.mark.parametrize("bits", [4, 8])
def test_dequant_formula_matches_reference(bits):
    w, s, b = GOLD[f"q{bits}_w"], GOLD[f"q{bits}_s"], GOLD[f"q{bits}_b"]
    K = w.shape[1] * 32 // bits
    ours = f32(O.dequantize(w, s, b, K, 64, bits))
    ref = GOLD[f"q{bits}_deq"]
    # oracle output is bf16(fma(s, q, b)); reference is fp32 q*s + b
    np.testing.assert_array_equal(O.f32_to_bf16(ref.astype(np.float32)), O.f32_to_bf16(ours))
    if bits == 4:
        np.testing.assert_array_equal(GOLD["q4_deq"], GOLD["q4_deq_l0"])


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_matches_reference_simulation(bits):
    w, s, b, x = GOLD[f"q{bits}_w"], GOLD[f"q{bits}_s"], GOLD[f"q{bits}_b"], GOLD["q4_x"]
    y = f32(O.qmm(x, w, s, b, bits))
    ref = GOLD[f"q{bits}_qmm"]
    # bf16 output: |err| <= half an ulp of the result plus fp32 reassociation
    tol = np.abs(ref) * 2.0**-8 + 1e-5 * np.max(np.abs(ref))
    assert np.all(np.abs(y - ref) <= tol)


def test_rms_norm_matches_reference():
    y = f32(O.rms_norm(GOLD["rms_x"], GOLD["rms_w"], 1e-6))
    ref = GOLD["rms_y"]
    assert np.all(np.abs(y - ref) <= np.abs(ref) * 2.0**-8 + 1e-6)


def test_argmax_known_answers():
    # tests/test_generate.cpp:21-36, 162-172 (first maximum wins)
    for vals, want in [([0.1, 0.3, 0.9, 0.2], 2), ([0.1, 0.5, 0.3], 1),
                       ([0.1, 0.2, 0.3, 10.0, 0.4], 3), ([0.5, 0.7, 0.7, 0.1], 1)]:
        l = O.f32_to_bf16(np.array([vals], np.float32))
        assert O.argmax(l)[0] == want


def test_exp_accuracy():
    L = O.lib()
    xs = np.linspace(-87, 88, 7001, dtype=np.float32)
    got = np.array([L.orc_exp(float(v)) for v in xs])
    rel = np.abs(got - np.exp(xs.astype(np.float64))) / np.exp(xs.astype(np.float64))
    assert rel.max() < 2e-7
    assert L.orc_exp(0.0) == 1.0


def test_rope_matches_reference_definition():
    # examples/test_device_rope.cpp:15-46: inv_freq = exp(i * (-ln(base)*2/dims)),
    # rx1 = x1 c - x2 s, rx2 = x2 c + x1 s.
    import ctypes as C
    L = O.lib()
    D, H, base = 128, 4, 1e6
    pos = np.array([0, 1, 17, 300, 4095], np.int32)
    x = O.gen_normal_bf16(1, 9, 1.0, len(pos) * H * D).reshape(len(pos), H, D)
    cos_t = np.empty((4096, D // 2), np.float32)
    sin_t = np.empty_like(cos_t)
    L.orc_rope_table(4096, D, base, O.ptr(cos_t), O.ptr(sin_t))
    y = x.copy()
    L.orc_rope(O.ptr(y), O.ptr(pos), len(pos), H, D, O.ptr(cos_t), O.ptr(sin_t))
    i = np.arange(D // 2, dtype=np.float32)
    inv = np.exp(i * np.float32(-math.log(base) * 2.0 / D)).astype(np.float32)
    th = pos[:, None].astype(np.float32) * inv[None, :]
    c, s = np.cos(th)[:, None, :], np.sin(th)[:, None, :]
    xf = f32(x)
    x1, x2 = xf[..., :D // 2], xf[..., D // 2:]
    ref = np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], -1)
    assert np.max(np.abs(f32(y) - ref)) < 2.0**-8 * np.max(np.abs(ref)) + 1e-3


def test_sdpa_matches_fp64_reference():
    # examples/test_sdpa_ref.cpp:81-100 style: fp64 softmax(q k^T s + mask) v
    L = O.lib()
    T, Hq, Hk, D, cap, off = 5, 4, 2, 128, 300, 250
    q = O.gen_normal_bf16(3, 1, 1.0, T * Hq * D)
    k = O.gen_normal_bf16(3, 2, 1.0, Hk * cap * D)
    v = O.gen_normal_bf16(3, 3, 1.0, Hk * cap * D)
    out = np.empty(T * Hq * D, np.uint16)
    scale = np.float32(1 / math.sqrt(D))
    L.orc_sdpa(O.ptr(q), O.ptr(k), O.ptr(v), O.ptr(out), T, Hq, Hk, D, cap, off, scale)
    qf = f32(q).reshape(T, Hq, D).astype(np.float64)
    kf = f32(k).reshape(Hk, cap, D).astype(np.float64)
    vf = f32(v).reshape(Hk, cap, D).astype(np.float64)
    o = f32(out).reshape(T, Hq, D)
    for t in range(T):
        for h in range(Hq):
            Lk = off + t + 1
            sc = kf[h // 2, :Lk] @ qf[t, h] * float(scale)
            p = np.exp(sc - sc.max())
            ref = (p / p.sum()) @ vf[h // 2, :Lk]
            assert np.max(np.abs(o[t, h] - ref)) < 2e-2


def test_sampler_exact_rules():
    L = O.lib()
    V = 1000
    logits = np.full(V, O.f32_to_bf16(np.float32(-5.0)), np.uint16)
    logits[17] = O.f32_to_bf16(np.float32(8.0))
    # top-p 0.5 keeps only the dominant token whatever the uniform
    for u in [0, 1, 2**23, 2**24 - 1]:
        assert L.orc_sample(O.ptr(logits), V, 0.7, 0.5, u) == 17
    # temperature 0 is argmax
    assert L.orc_sample(O.ptr(logits), V, 0.0, 1.0, 5) == 17
    # identical draft and target distributions accept every draft
    K = 4
    tl = O.gen_normal_bf16(5, 1, 1.0, (K + 1) * V).reshape(K + 1, V)
    drafts = np.array([3, 99, 500, 7], np.int32)
    ua = np.array([2**24 - 1] * K, np.uint32)
    out = np.empty(K + 1, np.int32)
    acc = L.orc_accept_stochastic(O.ptr(tl), O.ptr(tl[:K].copy()), O.ptr(drafts), K, V, 0.7, 1.0,
                                  O.ptr(ua), 123, O.ptr(out))
    assert acc == K and list(out[:K]) == list(drafts)
    # a draft with zero target mass (outside top-p) is always rejected
    tl2 = tl.copy()
    tl2[0, :] = O.f32_to_bf16(np.float32(-9.0))
    tl2[0, 11] = O.f32_to_bf16(np.float32(9.0))
    acc = L.orc_accept_stochastic(O.ptr(tl2), O.ptr(tl[:K].copy()), O.ptr(drafts), K, V, 0.7, 0.9,
                                  O.ptr(np.zeros(K, np.uint32)), 0, O.ptr(out))
    assert acc == 0 and out[0] == 11


def test_greedy_accept_rule():
    # src/common/generate.cpp:800-823: accept while argmax(logits[i]) == d_{i+1}
    L = O.lib()
    V, K = 50, 4
    preds = [4, 9, 2, 30, 8]
    tl = np.zeros((K + 1, V), np.uint16)
    for i, p in enumerate(preds):
        tl[i, p] = O.f32_to_bf16(np.float32(1.0))
    out = np.empty(K + 1, np.int32)
    assert L.orc_accept_greedy(O.ptr(tl), O.ptr(np.array([4, 9, 2, 30], np.int32)), K, V, O.ptr(out)) == 4
    assert list(out) == [4, 9, 2, 30, 8]  # bonus token
    assert L.orc_accept_greedy(O.ptr(tl), O.ptr(np.array([4, 7, 2, 30], np.int32)), K, V, O.ptr(out)) == 1
    assert list(out[:2]) == [4, 9]  # correction token


TINY = dict(hidden=256, layers=3, inter=512, heads=4, kv_heads=2, head_dim=128, vocab=1000,
            rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group=64)


@pytest.fixture(scope="module")
def tiny_model():
    L = O.lib()
    m = L.orc_model_create(O.ModelCfg(**TINY), 1234)
    yield m
    L.orc_model_free(m)


@pytest.mark.parametrize("kv_bits", [16, 8, 4])
def test_speculative_equals_plain_greedy(tiny_model, kv_bits):
    # exact mode: the verify block (B*(K+1) = 10 rows) and the single-row
    # decode steps of plain greedy take the same canonical order; with the
    # tensor-core paths on, blocks of >= 4 rows round differently and a
    # near-tie could flip a token
    L = O.lib()
    L.orc_set_mma_min_m(0)
    try:
        _speculative_vs_plain(L, tiny_model, kv_bits)
    finally:
        L.orc_set_mma_min_m(16)


def _speculative_vs_plain(L, tiny_model, kv_bits):
    B, P, MT = 2, 12, 30
    prompts = np.random.RandomState(1).randint(0, TINY["vocab"], (B, P)).astype(np.int32)
    spec = np.zeros((B, MT), np.int32)
    plain = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=4, max_tokens=MT, temperature=0.0, top_p=1.0, seed=0, draft_layers=1)
    assert L.orc_spec_generate(tiny_model, None, O.ptr(prompts), B, P, prm, kv_bits, O.ptr(spec),
                               O.ptr(st)) == 0
    assert L.orc_generate(tiny_model, O.ptr(prompts), B, P, MT, kv_bits, O.ptr(plain)) == 0
    np.testing.assert_array_equal(spec, plain)
    assert st[0] > 0 and st[1] >= st[2]


def test_emission_contract_first_token_is_prefill_argmax(tiny_model):
    # tests/test_generate.cpp:618-794: the token sampled by prepare() is emitted first
    L = O.lib()
    P = 9
    prompt = np.arange(P, dtype=np.int32)[None, :] * 7
    cache = L.orc_cache_create(tiny_model, TINY["layers"], 1, 64, 16)
    logits = np.zeros((P, TINY["vocab"]), np.uint16)
    assert L.orc_forward(tiny_model, cache, TINY["layers"], O.ptr(prompt), 1, P, O.ptr(logits)) == 0
    L.orc_cache_free(cache)
    first = O.argmax(logits[-1:])[0]
    out = np.zeros((1, 5), np.int32)
    assert L.orc_generate(tiny_model, O.ptr(prompt), 1, P, 5, 16, O.ptr(out)) == 0
    assert out[0, 0] == first


def test_set_position_rollback_is_exact(tiny_model):
    # tests/test_generate.cpp:854-870: set_position then re-append reproduces state
    L = O.lib()
    V = TINY["vocab"]
    cache = L.orc_cache_create(tiny_model, TINY["layers"], 1, 64, 16)
    toks = np.array([[5, 6, 7, 8, 9, 10]], np.int32)
    l1 = np.zeros((6, V), np.uint16)
    L.orc_forward(tiny_model, cache, TINY["layers"], O.ptr(toks), 1, 6, O.ptr(l1))
    extra = np.array([[44, 45, 46]], np.int32)
    lx = np.zeros((3, V), np.uint16)
    L.orc_forward(tiny_model, cache, TINY["layers"], O.ptr(extra), 1, 3, O.ptr(lx))
    assert L.orc_cache_len(cache, 0) == 9
    L.orc_cache_set_position(cache, 0, 6)
    ly = np.zeros((3, V), np.uint16)
    L.orc_forward(tiny_model, cache, TINY["layers"], O.ptr(extra), 1, 3, O.ptr(ly))
    np.testing.assert_array_equal(lx, ly)
    L.orc_cache_free(cache)


def test_kv_quirk_allocation_rule():
    # the reference's KVCacheSimple allocation after a prompt of n tokens
    # (512-token chunks while more remain; first allocation max(chunk, 256);
    # doubling when a chunk does not fit): kv_cache.cpp:34-110, llm_model.h:18-60
    L = O.lib()
    for n, want in [(1, 256), (40, 256), (255, 256), (256, 256), (257, 257), (300, 300), (512, 512),
                    (513, 1024), (600, 1024), (1100, 2048), (8192, 8192)]:
        assert L.orc_kv_quirk_alloc(n) == want, (n, L.orc_kv_quirk_alloc(n), want)
