"""Host side of tensor parallelism, on the CPU: the handle exchange over a
2-rank gloo group, and the oracle's tensor-parallel emulation and synthetic
context (the checkers the 2-GPU parity test relies on)."""
import ctypes as C
import datetime
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle_lib as O
from conftest import load_lmx

SMALL = dict(hidden=512, layers=2, inter=1024, heads=8, kv_heads=4, head_dim=128, vocab=2048,
             rope_theta=5e5, eps=1e-5, qk_norm=0, tied=0, bits=4, group=64)


def _exchange_rank(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    lmx = load_lmx()
    got = lmx.exchange_handles(bytes([rank + 1]) * lmx.TP_HANDLE_BYTES)
    ok = got == [bytes([r + 1]) * lmx.TP_HANDLE_BYTES for r in range(world)]
    bad_raised = False
    try:  # a short handle from any rank is rejected on every rank
        lmx.exchange_handles(b"x" * (lmx.TP_HANDLE_BYTES - (rank == 1)))
    except lmx.LmxError:
        bad_raised = True
    with open(os.path.join(outdir, f"r{rank}"), "w") as f:
        f.write(f"{int(ok)} {int(bad_raised)}")
    dist.destroy_process_group()


def test_handle_exchange_gloo_world2(tmp_path):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_exchange_rank, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        assert (tmp_path / f"r{r}").read_text() == "1 1"


def _forward(o, tp, tokens, kv_bits=8, ctx=0):
    assert O.lib().orc_model_set_tp(o, tp) == 0
    B, T = tokens.shape
    oc = O.lib().orc_cache_create(o, SMALL["layers"], B, 64, kv_bits)
    if ctx:
        assert O.lib().orc_cache_fill_synthetic(oc, ctx, 3, 0x40000000) == 0
    out = np.zeros((B, T, SMALL["vocab"]), np.uint16)
    assert O.lib().orc_forward(o, oc, SMALL["layers"], O.ptr(tokens), B, T, O.ptr(out)) == 0
    lens = [O.lib().orc_cache_len(oc, b) for b in range(B)]
    O.lib().orc_cache_free(oc)
    return out, lens


@pytest.fixture(scope="module")
def small_model():
    O.lib().orc_set_mma_min_m(0)
    o = O.lib().orc_model_create(C.byref(O.ModelCfg(**SMALL)), 5)
    yield o
    O.lib().orc_model_free(o)
    O.lib().orc_set_mma_min_m(16)


def test_oracle_tp_emulation_close_to_unsplit(small_model):
    tok = np.random.RandomState(1).randint(0, SMALL["vocab"], (2, 6)).astype(np.int32)
    ref, _ = _forward(small_model, 1, tok, ctx=20)
    again, _ = _forward(small_model, 1, tok, ctx=20)
    np.testing.assert_array_equal(ref, again)
    r = O.bf16_to_f32(ref)
    for tp in (2, 4):
        got, lens = _forward(small_model, tp, tok, ctx=20)
        assert lens == [26, 26]
        g = O.bf16_to_f32(got)
        # a different fp32 summation order only: well inside the contract
        assert np.abs(g - r).max() < 2e-2 + 2.0 ** -7 * np.abs(r).max()
        assert (got != ref).any() or tp == 1
    assert O.lib().orc_model_set_tp(small_model, 3) != 0  # heads 8 % 3
    assert O.lib().orc_model_set_tp(small_model, 1) == 0


def test_oracle_synthetic_context_is_standard_normal():
    cfg = dict(SMALL, layers=1)
    o = O.lib().orc_model_create(C.byref(O.ModelCfg(**cfg)), 5)
    oc = O.lib().orc_cache_create(o, 1, 2, 512, 16)
    assert O.lib().orc_cache_fill_synthetic(oc, 500, 8, 0x40000000) == 0
    assert O.lib().orc_cache_fill_synthetic(oc, 513, 8, 0x40000000) != 0  # > capacity
    assert [O.lib().orc_cache_len(oc, b) for b in range(2)] == [500, 500]
    # the fill draws layer 0's K from the Philox normal of tensor 0x40000000
    # (elements ((b*Hk + hk)*rows + j)*128 + d); that draw is N(0, 1)
    Hk, rows = cfg["kv_heads"], 500
    vals = O.gen_normal_bf16(8, 0x40000000, 1.0, 2 * Hk * rows * 128)
    v = O.bf16_to_f32(vals)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01
    O.lib().orc_cache_free(oc)
    O.lib().orc_model_free(o)
