"""K3 on the B200 vs the oracle: temperature / top-p sampling, rejection
sampling and the stochastic speculative stream.  Decisions are exact integer
comparisons on both sides, so the bar is equality."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu


def dev(cuda, a):
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, None)
    return cuda.from_numpy(np.ascontiguousarray(a.view(view) if view else a)).cuda()


def logits_cases(rng, V):
    yield O.gen_normal_bf16(rng.randint(1 << 30), 1, 1.0, V)
    tied = np.full(V, O.f32_to_bf16(np.float32(-3.0)), np.uint16)  # many exact ties
    tied[rng.choice(V, V // 4, replace=False)] = O.f32_to_bf16(np.float32(1.0))
    tied[rng.choice(V, 7, replace=False)] = O.f32_to_bf16(np.float32(2.5))
    yield tied
    peaked = O.gen_normal_bf16(rng.randint(1 << 30), 2, 0.3, V)
    peaked[V // 2] = O.f32_to_bf16(np.float32(9.0))
    yield peaked


@pytest.mark.parametrize("V", [1000, 151936])
@pytest.mark.parametrize("temperature,top_p", [(0.7, 0.9), (1.0, 1.0), (0.5, 0.3), (1.3, 0.999), (0.7, 0.0001)])
def test_sample_matches_oracle(lmx, cuda, V, temperature, top_p):
    rng = np.random.RandomState(V + int(temperature * 10) + int(top_p * 100))
    rows = list(logits_cases(rng, V))
    L = np.stack(rows)
    us = np.array([0, 2**24 - 1, 123456, 8388608, 999], np.uint32)
    for u in us:
        u24 = np.full(len(rows), u, np.uint32)
        out = cuda.empty(len(rows), dtype=cuda.int32, device="cuda")
        dl, du = dev(cuda, L), dev(cuda, u24)
        lmx.call("lmx_sample", dl.data_ptr(), len(rows), V, temperature, top_p, du.data_ptr(), out.data_ptr(), None)
        got = out.cpu().numpy()
        for r in range(len(rows)):
            ref = O.lib().orc_sample(O.ptr(np.ascontiguousarray(L[r])), V, temperature, top_p, int(u))
            assert got[r] == ref, (r, int(u), got[r], ref)


@pytest.mark.parametrize("V,top_p", [(1000, 0.9), (1000, 1.0), (151936, 0.9)])
def test_spec_accept_matches_oracle(lmx, cuda, V, top_p):
    rng = np.random.RandomState(V + int(top_p * 10))
    B, K, T = 6, 5, 0.7
    tl = O.gen_normal_bf16(11, V, 1.0, B * (K + 1) * V).reshape(B, K + 1, V)
    ql = O.gen_normal_bf16(12, V, 1.0, B * K * V).reshape(B, K, V)
    # sequence 1: identical p and q (every draft accepted, bonus drawn);
    # sequence 2: target mass concentrated away from the drafts (reject at 0)
    ql[1] = tl[1, :K]
    tl[2, :, :] = O.f32_to_bf16(np.float32(-8.0))
    tl[2, :, 5] = O.f32_to_bf16(np.float32(8.0))
    drafts = np.zeros((B, K), np.int32)
    for b in range(B):
        for i in range(K):
            drafts[b, i] = O.lib().orc_sample(O.ptr(np.ascontiguousarray(ql[b, i])), V, T, top_p,
                                              int(rng.randint(1 << 24)))
    drafts[2, 0] = 6
    ua = rng.randint(0, 1 << 24, (B, K)).astype(np.uint32)
    uf = rng.randint(0, 1 << 24, B).astype(np.uint32)
    nacc = cuda.empty(B, dtype=cuda.int32, device="cuda")
    outt = cuda.full((B, K + 1), -1, dtype=cuda.int32, device="cuda")
    # keep every device tensor referenced until the kernel has run (a temporary
    # would go back to the caching allocator and be reused by the next upload)
    dt, dq, dd, dua, duf = dev(cuda, tl), dev(cuda, ql), dev(cuda, drafts), dev(cuda, ua), dev(cuda, uf)
    lmx.call("lmx_spec_accept", dt.data_ptr(), dq.data_ptr(), dd.data_ptr(), B, K, V, T, top_p,
             dua.data_ptr(), duf.data_ptr(), nacc.data_ptr(), outt.data_ptr(), None)
    cuda.cuda.synchronize()
    got_n, got_t = nacc.cpu().numpy(), outt.cpu().numpy()
    seen = set()
    for b in range(B):
        ref = np.zeros(K + 1, np.int32)
        n = O.lib().orc_accept_stochastic(O.ptr(np.ascontiguousarray(tl[b])), O.ptr(np.ascontiguousarray(ql[b])),
                                          O.ptr(np.ascontiguousarray(drafts[b])), K, V, T, top_p,
                                          O.ptr(np.ascontiguousarray(ua[b])), int(uf[b]), O.ptr(ref))
        assert got_n[b] == n, (b, got_n[b], n)
        np.testing.assert_array_equal(got_t[b, :n + 1], ref[:n + 1])
        seen.add(n)
    assert got_n[1] == K and got_n[2] == 0


TINY = dict(hidden=512, layers=3, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=1000,
            rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)


@pytest.mark.parametrize("kv_bits,top_p,B,K", [(16, 0.9, 3, 4), (4, 1.0, 3, 4), (4, 0.9, 8, 5)])
def test_stochastic_spec_stream_matches_oracle(lmx, cuda, mma_threshold, kv_bits, top_p, B, K):
    # exact mode (canonical matmul order everywhere): identical streams; the
    # last case has config 3's batch 8, K = 5, 4-bit KV, T 0.7, top-p 0.9
    mma_threshold(0)
    P, MT, T, seed = 20, 40, 0.7, 77
    g = lmx.Model(TINY, 4321)
    ocfg = dict(TINY)
    ocfg["group"] = ocfg.pop("group_size")
    o = O.lib().orc_model_create(C.byref(O.ModelCfg(**ocfg)), 4321)
    prompts = np.random.RandomState(9).randint(0, TINY["vocab"], (B, P)).astype(np.int32)
    sd = lmx.SpecDecoder(g, None, 1, B, K, MT, P, kv_bits=kv_bits, temperature=T, top_p=top_p, seed=seed)
    sd.prefill(prompts)
    sd.decode(use_graph=True)
    got, stats = sd.result()
    sd.close()
    g.close()
    ref = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=K, max_tokens=MT, temperature=T, top_p=top_p, seed=seed, draft_layers=1)
    assert O.lib().orc_spec_generate(o, None, O.ptr(prompts), B, P, prm, kv_bits, O.ptr(ref), O.ptr(st)) == 0
    O.lib().orc_model_free(o)
    np.testing.assert_array_equal(got, ref)
    assert stats["accepted"] == st[2]


def test_separate_draft_other_gqa_stream_matches_oracle(lmx, cuda, mma_threshold):
    # config 3's structure at test size: a separate draft model whose width,
    # head count and KV-head count differ from the target's (one workspace
    # serves both), batch 8, K = 5, 4-bit KV, T 0.7, top-p 0.9; exact mode
    mma_threshold(0)
    draft_cfg = dict(TINY, hidden=512, layers=2, inter=512, heads=8, kv_heads=1)
    B, P, K, MT, T, tp, seed = 8, 20, 5, 30, 0.7, 0.9, 5
    g = lmx.Model(TINY, 111)
    gd = lmx.Model(draft_cfg, 222)

    def ocfg(c):
        d = dict(c)
        d["group"] = d.pop("group_size")
        return O.ModelCfg(**d)

    o = O.lib().orc_model_create(C.byref(ocfg(TINY)), 111)
    od = O.lib().orc_model_create(C.byref(ocfg(draft_cfg)), 222)
    prompts = np.random.RandomState(13).randint(0, TINY["vocab"], (B, P)).astype(np.int32)
    sd = lmx.SpecDecoder(g, gd, draft_cfg["layers"], B, K, MT, P, kv_bits=4, temperature=T, top_p=tp, seed=seed)
    sd.prefill(prompts)
    sd.decode(use_graph=True)
    got, stats = sd.result()
    sd.close()
    g.close()
    gd.close()
    ref = np.zeros((B, MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=K, max_tokens=MT, temperature=T, top_p=tp, seed=seed, draft_layers=draft_cfg["layers"])
    assert O.lib().orc_spec_generate(o, od, O.ptr(prompts), B, P, prm, 4, O.ptr(ref), O.ptr(st)) == 0
    O.lib().orc_model_free(o)
    O.lib().orc_model_free(od)
    np.testing.assert_array_equal(got, ref)
    assert stats["accepted"] == st[2]
