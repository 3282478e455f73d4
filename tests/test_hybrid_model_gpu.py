"""Configuration 4 end to end on the B200 vs the oracle (exact mode, every
matmul in the canonical order): the hybrid trunk's logits over prefill and
decode blocks (Gated DeltaNet states, conv windows and attention caches
carried across calls), and the MTP speculative stream (2 drafts per step,
greedy; cache rollback and Gated DeltaNet state commit at the accepted
prefix) -- bit-identical.  Tensor-core mode is not compared on this model:
its top-k expert routing is discontinuous, so a one-ulp router difference
can select a different expert."""
import ctypes as C

import numpy as np
import pytest

import hybrid_cases as H
import oracle_lib as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def hybrid(lmx, cuda):
    cfg = H.TINY_HYBRID
    h = C.c_void_p()
    lmx.call("lmx_hybrid_create", C.byref(lmx.HybridConfig(**cfg)), 77, C.byref(h))
    o = H.oracle_hybrid(cfg, 77)
    yield cfg, h, o
    lmx.lib().lmx_hybrid_free(h)
    O.lib().orc_hybrid_free(o)


@pytest.mark.parametrize("kv_bits", [16, 8])
def test_hybrid_forward_logits_bit_exact(lmx, hybrid, mma_threshold, kv_bits):
    mma_threshold(0)
    cfg, h, o = hybrid
    B, V = 2, cfg["vocab"]
    rng = np.random.RandomState(kv_bits)
    blocks = [rng.randint(0, V, (B, T)).astype(np.int32) for T in (37, 5, 1, 3)]
    ref = H.oracle_hybrid_forward_blocks(o, cfg, B, 96, kv_bits, blocks)
    st = C.c_void_p()
    lmx.call("lmx_hybrid_state_create", h, B, 96, kv_bits, 40, C.byref(st))
    for i, tok in enumerate(blocks):
        T = tok.shape[1]
        lg = np.zeros((B, T, V), np.uint16)
        lmx.call("lmx_hybrid_forward", h, st, tok.ctypes.data, B, T, lg.ctypes.data)
        bad = np.argwhere(lg != ref[i])
        assert bad.size == 0, f"block {i}: {len(bad)} mismatching logits, first {bad[:3].tolist()}"
    lmx.lib().lmx_hybrid_state_free(st)


@pytest.mark.parametrize("use_graph", [True, False])
def test_hybrid_mtp_stream_matches_oracle(lmx, hybrid, mma_threshold, use_graph):
    mma_threshold(0)
    cfg, h, o = hybrid
    B, P, MT = 3, 20, 24
    prompts = np.random.RandomState(5).randint(0, cfg["vocab"], (B, P)).astype(np.int32)
    ref, rst = H.oracle_hybrid_spec(o, prompts, MT, 16)
    sp = C.c_void_p()
    lmx.call("lmx_hybrid_spec_create", h, B, MT, P, 16, C.byref(sp))
    lmx.call("lmx_hybrid_spec_prefill", sp, prompts.ctypes.data)
    sec = C.c_double()
    lmx.call("lmx_hybrid_spec_decode", sp, 1 if use_graph else 0, C.byref(sec))
    out = np.zeros((B, MT), np.int32)
    stats = np.zeros(5, np.int64)
    lmx.call("lmx_hybrid_spec_result", sp, out.ctypes.data, stats.ctypes.data)
    lmx.lib().lmx_hybrid_spec_free(sp)
    np.testing.assert_array_equal(out, ref)
    assert stats[0] == rst[0] and stats[2] == rst[2] and stats[3] == rst[3]
