"""The reference's generate / TokenIterator contract over the speculative
decoder (src/common/generate.cpp:968-1045, :1061-1125; include/mlx-lm/common/
generate.h:170-228): per-token next() in emission order, max_tokens, EOS
(ends a sequence, not counted), the cancellation predicate polled before
every step, a callback that stops its sequence, the completion counters, and
the plain-decode fallback (K = 0).  Exact mode, so every stream is checked
token for token against the oracle."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, layers=3, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=1000,
           rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)
B, P, K, MT = 2, 20, 4, 40


@pytest.fixture(scope="module")
def setup(lmx, cuda):
    g = lmx.Model(CFG, 1234)
    ocfg = dict(CFG)
    ocfg["group"] = ocfg.pop("group_size")
    o = O.lib().orc_model_create(C.byref(O.ModelCfg(**ocfg)), 1234)
    prompts = np.random.RandomState(7).randint(0, CFG["vocab"], (B, P)).astype(np.int32)
    ref = np.zeros((B, MT), np.int32)
    O.lib().orc_set_mma_min_m(0)
    assert O.lib().orc_generate(o, O.ptr(prompts), B, P, MT, 16, O.ptr(ref)) == 0
    O.lib().orc_set_mma_min_m(16)
    yield g, prompts, ref
    g.close()
    O.lib().orc_model_free(o)


@pytest.mark.parametrize("k", [K, 0])
def test_next_streams_equal_reference_greedy(lmx, setup, mma_threshold, k):
    # k = 0: plain decoding, one token per step (the reference's fallback)
    g, prompts, ref = setup
    mma_threshold(0)
    sd = lmx.SpecDecoder(g, None, 1, B, k, MT, P, kv_bits=16)
    sd.prefill(prompts)
    got = [[] for _ in range(B)]
    while True:
        t = sd.next()
        if t is None:
            break
        for b in range(B):
            if t[b] >= 0:
                got[b].append(int(t[b]))
    out, st = sd.result()
    sd.close()
    np.testing.assert_array_equal(np.array(got), ref)
    np.testing.assert_array_equal(out, ref)
    if k == 0:
        assert st["steps"] == B * MT and st["accepted"] == 0


def test_generate_eos_cancel_and_callback(lmx, setup, mma_threshold):
    g, prompts, ref = setup
    mma_threshold(0)
    sd = lmx.SpecDecoder(g, None, 1, B, K, MT, P, kv_bits=16)
    # EOS: sequence 0's 10th token; it ends that sequence without being
    # counted or passed on (unless it occurred earlier in the stream)
    eos = int(ref[0, 10])
    first = {b: next((i for i in range(MT) if ref[b, i] == eos), MT) for b in range(B)}
    seen = {b: [] for b in range(B)}
    info = sd.generate(prompts, eos=[eos], on_token=lambda b, t: seen[b].append(t) and False)
    for b in range(B):
        assert seen[b] == list(ref[b, :first[b]])
        assert info[b].generation_token_count == first[b]
        assert info[b].prompt_token_count == P
        assert info[b].mtp_draft_tokens_proposed == K * info[b].mtp_speculative_steps
        assert info[b].prompt_time > 0
    # on_token stop: each sequence stops after its 5th token
    seen = {b: [] for b in range(B)}
    info = sd.generate(prompts, on_token=lambda b, t: (seen[b].append(t), len(seen[b]) >= 5)[1])
    for b in range(B):
        assert seen[b] == list(ref[b, :5]) and info[b].generation_token_count == 5
    # cancellation before the forward passes: polled before every step
    polls = [0]

    def cancel():
        polls[0] += 1
        return polls[0] > 3

    seen = {b: [] for b in range(B)}
    info = sd.generate(prompts, should_cancel=cancel, on_token=lambda b, t: seen[b].append(t) and False)
    assert polls[0] == 4
    for b in range(B):
        assert 1 <= len(seen[b]) < MT and seen[b] == list(ref[b, :len(seen[b])])
    sd.close()
