"""The oracle's hybrid-model ops (configuration 4) against float64
restatements of the reference formulas (tests/hybrid_cases.py): the canonical
orders may round differently, but the math must be the reference's."""
import numpy as np
import pytest

import hybrid_cases as H
import oracle_lib as O


def test_log_matches_libm():
    xs = np.concatenate([np.geomspace(1e-30, 1e30, 2001), np.linspace(0.5, 2.0, 1001)]).astype(np.float32)
    got = np.array([O.lib().orc_log(float(x)) for x in xs], np.float64)
    ref = np.log(xs.astype(np.float64))
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)
    assert err.max() < 4e-7, err.max()


@pytest.mark.parametrize("Hk,Hv", [(2, 4), (1, 1)])
def test_gdn_oracle_matches_reference_math(Hk, Hv):
    c = H.gdn_case(3 + Hv, B=2, T=3, Hk=Hk, Hv=Hv)
    out, snap = H.oracle_gdn(c)
    ref_out, ref_state = H.reference_gdn(c)
    g = O.bf16_to_f32(out)
    # bf16 rounding after conv, SiLU, the q/k norms and y: a few bf16 ulps
    assert np.abs(g - ref_out).max() < 3e-2 + 2e-2 * np.abs(ref_out).max()
    assert np.abs(snap[:, -1] - ref_state).max() < 2e-2 * max(1.0, np.abs(ref_state).max())


def test_gdn_commit_selects_state_and_window():
    c = H.gdn_case(11, B=3, T=4, Hk=1, Hv=2)
    _, snap = H.oracle_gdn(c)
    acc = np.array([0, 3, 1], np.int32)
    state, conv = H.oracle_commit(c, snap, acc)
    win = np.concatenate([c["conv_state"], c["qkv"]], 1)  # [B, 3+T, CD]
    for b, t in enumerate(acc):
        np.testing.assert_array_equal(state[b], snap[b, t])
        np.testing.assert_array_equal(conv[b], win[b, t + 1:t + 4])


def test_moe_route_oracle_topk_softmax():
    logits = H.moe_route_case(5, rows=12, E=512)
    idx, w = H.oracle_route(logits, 10)
    l = O.bf16_to_f32(logits)
    for r in range(12):
        order = sorted(range(512), key=lambda e: (-l[r, e], e))[:10]
        assert list(idx[r]) == order
        top = l[r, order].astype(np.float64)
        p = np.exp(top - top.max())
        np.testing.assert_allclose(w[r], p / p.sum(), rtol=2e-6, atol=1e-7)
    assert idx[0][0] == 5 and idx[0][1] == 7  # the tie: lower index first


@pytest.mark.parametrize("bits", [4, 8])
def test_moe_experts_oracle_matches_dequant_matmul(bits):
    c = H.moe_experts_case(7 + bits, M=3, H=512, I=512, E=6, k=3, bits=bits)
    got = O.bf16_to_f32(H.oracle_experts(c))
    ref = H.reference_experts(c)
    # bf16 rounding of gate / up / act / each expert's output
    assert np.abs(got - ref).max() < 2e-2 * np.abs(ref).max() + 1e-2


def test_hybrid_oracle_block_equals_token_by_token():
    # exact mode: a forward over a 6-token block and six single-token
    # forwards give the same logits (attention cache, Gated DeltaNet state
    # and conv window carried across calls, MoE per row) -- with fp32 states:
    # the reference's bf16 states (the default) are rounded between blocks
    # but not within one, so there the two differ by design
    O.lib().orc_set_mma_min_m(0)
    O.lib().orc_set_gdn_state_bf16(0)
    cfg = H.TINY_HYBRID
    o = H.oracle_hybrid(cfg, 9)
    tok = np.random.RandomState(2).randint(0, cfg["vocab"], (2, 10)).astype(np.int32)
    pre = tok[:, :4]
    blk = H.oracle_hybrid_forward_blocks(o, cfg, 2, 32, 8, [pre, tok[:, 4:]])[1]
    one = H.oracle_hybrid_forward_blocks(o, cfg, 2, 32, 8, [pre] + [tok[:, i:i + 1] for i in range(4, 10)])[1:]
    for i in range(6):
        np.testing.assert_array_equal(blk[:, i], one[i][:, 0])
    O.lib().orc_hybrid_free(o)
    O.lib().orc_set_mma_min_m(16)
    O.lib().orc_set_gdn_state_bf16(1)
