"""REF_KV_PAD_QUIRK: the reference's maybe_quantize_kv_cache (src/common/
kv_cache.cpp:391-413) prefills the prompt with a bf16 cache, then quantizes
the whole allocation -- zero rows past the prompt included -- and decodes on
from the allocation length.  The engine's quirk mode against the oracle's,
exact mode: speculative greedy streams identical token for token; and the
quirk changes the stream when the allocation pads the prompt."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, layers=3, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=1000,
           rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)


@pytest.mark.parametrize("kv_bits", [4, 8])
@pytest.mark.parametrize("P", [40, 300])
def test_quirk_stream_matches_oracle(lmx, cuda, mma_threshold, kv_bits, P):
    # P = 40 pads to a 256-row allocation; P = 300 to 300 (one chunk), so
    # only the bf16 prefill differs from the intended semantics
    mma_threshold(0)
    B, K, MT = 2, 4, 24
    g = lmx.Model(CFG, 1234)
    ocfg = dict(CFG)
    ocfg["group"] = ocfg.pop("group_size")
    o = O.lib().orc_model_create(C.byref(O.ModelCfg(**ocfg)), 1234)
    prompts = np.random.RandomState(P).randint(0, CFG["vocab"], (B, P)).astype(np.int32)
    streams = {}
    try:
        for quirk in (0, 1):
            sd = lmx.SpecDecoder(g, None, 1, B, K, MT, P, kv_bits=kv_bits, kv_quirk=quirk)
            sd.prefill(prompts)
            sd.decode()
            got, _ = sd.result()
            sd.close()
            O.lib().orc_set_kv_quirk(quirk)
            ref = np.zeros((B, MT), np.int32)
            st = np.zeros(5, np.int64)
            prm = O.SpecParams(K=K, max_tokens=MT, temperature=0.0, top_p=1.0, seed=0, draft_layers=1)
            assert O.lib().orc_spec_generate(o, None, O.ptr(prompts), B, P, prm, kv_bits, O.ptr(ref), O.ptr(st)) == 0
            np.testing.assert_array_equal(got, ref)
            streams[quirk] = got
    finally:
        O.lib().orc_set_kv_quirk(0)
        g.close()
        O.lib().orc_model_free(o)
    if O.lib().orc_kv_quirk_alloc(P) > P:  # zero rows enter attention and RoPE positions jump
        assert not np.array_equal(streams[0], streams[1])
