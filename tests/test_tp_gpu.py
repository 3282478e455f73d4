"""Tensor parallelism on 2 GPUs (one process per GPU) vs the oracle's
tensor-parallel emulation: the same shards, partials summed in fp32 in rank
order.  Exact mode: logits and the greedy stream bit-identical.  Tensor-core
mode: logits within the numerics contract's tolerance."""
import ctypes as C
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import checkpoint_io as CK
import oracle_lib as O
import tp_worker as W

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def oracle_cfg(cfg):
    d = dict(cfg)
    d["group"] = d.pop("group_size")
    return O.ModelCfg(**d)


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.fixture(scope="module")
def tp2_result(cuda, tmp_path_factory):
    if cuda.cuda.device_count() < 2:
        pytest.skip("tensor-parallel test needs 2 GPUs")
    tmp = tmp_path_factory.mktemp("tp")
    out = str(tmp / "tp2.npz")
    ckpt = str(tmp / "ckpt")
    make_tp_checkpoint(ckpt)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(HERE, "tp_worker.py"), "--out", out, "--ckpt", ckpt]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, f"tp worker failed:\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    res = dict(np.load(out))
    res["ckpt"] = ckpt
    return res


# Qwen3-style 4-bit checkpoint with 8-bit overrides on a row-split (o_proj),
# a column-split (gate/up) layer and the vocab-split lm_head
CKPT_CFG = dict(W.TARGET, qk_norm=1, group=64, rope_factor=0.0, rope_low_freq=0.0, rope_high_freq=0.0,
                rope_orig_max_pos=0.0)
del CKPT_CFG["group_size"]
CKPT_OVER = {"model.layers.0.self_attn.o_proj": 8, "model.layers.1.mlp.gate_proj": 8,
             "model.layers.1.mlp.up_proj": 8, "lm_head": 8}


def make_tp_checkpoint(d):
    CK.make_checkpoint(d, CKPT_CFG, 77, overrides=CKPT_OVER)


def oracle_forward_logits(tp, mma):
    O.lib().orc_set_mma_min_m(mma)
    cfg = W.TARGET_TIED8
    o = O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), W.SEED)
    assert O.lib().orc_model_set_tp(o, tp) == 0
    oc = O.lib().orc_cache_create(o, cfg["layers"], W.B, 128, 8)
    assert O.lib().orc_cache_fill_synthetic(oc, W.CTX, W.CTX_SEED, 0x40000000) == 0
    outs = []
    for tok in W.forward_tokens():
        T = tok.shape[1]
        ol = np.zeros((W.B, T, cfg["vocab"]), np.uint16)
        assert O.lib().orc_forward(o, oc, cfg["layers"], O.ptr(tok), W.B, T, O.ptr(ol)) == 0
        outs.append(ol)
    O.lib().orc_cache_free(oc)
    O.lib().orc_model_free(o)
    O.lib().orc_set_mma_min_m(16)
    return outs


def test_tp2_forward_logits_bit_exact(tp2_result):
    for i, ref in enumerate(oracle_forward_logits(2, 0)):
        got = tp2_result[f"logits_mma0_{i}"]
        bad = np.argwhere(got != ref)
        assert bad.size == 0, f"block {i}: {len(bad)} mismatching logits, first {bad[:3].tolist()}"


def test_tp2_forward_logits_tensor_core(tp2_result):
    for i, ref in enumerate(oracle_forward_logits(2, 16)):
        g, r = O.bf16_to_f32(tp2_result[f"logits_mma16_{i}"]), O.bf16_to_f32(ref)
        tol = 2e-2 + np.abs(r) * 2.0 ** -7
        assert not (np.abs(g - r) > tol).any(), f"block {i}: max |diff| {np.abs(g - r).max():.4g}"


def test_tp2_greedy_stream_matches_oracle(tp2_result):
    O.lib().orc_set_mma_min_m(0)
    to = O.lib().orc_model_create(C.byref(oracle_cfg(W.TARGET)), W.SEED)
    do = O.lib().orc_model_create(C.byref(oracle_cfg(W.DRAFT)), W.SEED + 1)
    assert O.lib().orc_model_set_tp(to, 2) == 0
    p = W.prompts()
    out = np.zeros((W.B, W.MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=W.K, max_tokens=W.MT, temperature=0.0, top_p=1.0, seed=0, draft_layers=1,
                       context_len=W.CTX, context_seed=W.CTX_SEED)
    rc = O.lib().orc_spec_generate(to, do, O.ptr(p), W.B, W.P, prm, 8, O.ptr(out), O.ptr(st))
    O.lib().orc_model_free(to)
    O.lib().orc_model_free(do)
    O.lib().orc_set_mma_min_m(16)
    assert rc == 0
    np.testing.assert_array_equal(tp2_result["stream"], out)
    assert int(tp2_result["accepted"]) == st[2]


def test_tp2_checkpoint_shards_bit_exact(tp2_result):
    # each rank copied only its block of every tensor; together they give
    # the oracle's tensor-parallel emulation of the whole checkpoint
    O.lib().orc_set_mma_min_m(0)
    cfg, o = CK.oracle_from_checkpoint(tp2_result["ckpt"])
    assert O.lib().orc_model_set_tp(o, 2) == 0
    oc = O.lib().orc_cache_create(o, cfg["layers"], W.B, 128, 16)
    try:
        for i, tok in enumerate(W.forward_tokens()):
            T = tok.shape[1]
            ol = np.zeros((W.B, T, cfg["vocab"]), np.uint16)
            assert O.lib().orc_forward(o, oc, cfg["layers"], O.ptr(tok), W.B, T, O.ptr(ol)) == 0
            got = tp2_result[f"ckpt_logits_{i}"]
            bad = np.argwhere(got != ol)
            assert bad.size == 0, f"block {i}: {len(bad)} mismatching logits, first {bad[:3].tolist()}"
    finally:
        O.lib().orc_cache_free(oc)
        O.lib().orc_model_free(o)
        O.lib().orc_set_mma_min_m(16)


def test_tp2_sharded_draft_stream_matches_oracle(tp2_result):
    # the draft as a tensor-parallel shard too (vocab-parallel draft argmax):
    # the oracle emulates the split in both models
    O.lib().orc_set_mma_min_m(0)
    to = O.lib().orc_model_create(C.byref(oracle_cfg(W.TARGET)), W.SEED)
    do = O.lib().orc_model_create(C.byref(oracle_cfg(W.DRAFT)), W.SEED + 1)
    assert O.lib().orc_model_set_tp(to, 2) == 0
    assert O.lib().orc_model_set_tp(do, 2) == 0
    p = W.prompts()
    out = np.zeros((W.B, W.MT), np.int32)
    st = np.zeros(5, np.int64)
    prm = O.SpecParams(K=W.K, max_tokens=W.MT, temperature=0.0, top_p=1.0, seed=0, draft_layers=1,
                       context_len=W.CTX, context_seed=W.CTX_SEED)
    rc = O.lib().orc_spec_generate(to, do, O.ptr(p), W.B, W.P, prm, 8, O.ptr(out), O.ptr(st))
    O.lib().orc_model_free(to)
    O.lib().orc_model_free(do)
    O.lib().orc_set_mma_min_m(16)
    assert rc == 0
    np.testing.assert_array_equal(tp2_result["stream_tp_draft"], out)
    assert int(tp2_result["accepted_tp_draft"]) == st[2]
