"""Hybrid-model ops (configuration 4) on the B200 vs the oracle, through the
C ABI: Gated DeltaNet verify step (output and every per-token state
bit-identical), its commit / rollback, the MoE router and the routed
experts (bit-identical)."""
import ctypes as C

import numpy as np
import pytest

import hybrid_cases as H
import oracle_lib as O

pytestmark = pytest.mark.gpu


def dev(cuda, a):
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, None)
    return cuda.from_numpy(np.ascontiguousarray(a.view(view) if view else a)).cuda()


def host(t, dtype):
    a = t.cpu().numpy()
    return a.view(dtype) if a.dtype != dtype else a


def gdn_device(lmx, cuda, c):
    B, T, Hk, Hv = c["B"], c["T"], c["Hk"], c["Hv"]
    d = {k: dev(cuda, c[k]) for k in ("qkv", "z", "b", "a", "conv_w", "a_log", "dt_bias", "norm_w",
                                      "conv_state", "state")}
    d["snap"] = cuda.zeros((B, T, Hv, 128, 128), dtype=cuda.float32, device="cuda")
    d["out"] = cuda.zeros((B, T, Hv * 128), dtype=cuda.int16, device="cuda")
    d["scratch"] = cuda.zeros(lmx.lib().lmx_gdn_scratch_bytes(B, T, Hk, Hv), dtype=cuda.uint8, device="cuda")
    g = lmx.GdnDesc(batch=B, T=T, k_heads=Hk, v_heads=Hv, eps=c["eps"])
    for f, k in (("qkv", "qkv"), ("z", "z"), ("b", "b"), ("a", "a"), ("conv_w", "conv_w"), ("a_log", "a_log"),
                 ("dt_bias", "dt_bias"), ("norm_w", "norm_w"), ("conv_state", "conv_state"), ("state", "state"),
                 ("state_snap", "snap"), ("out", "out"), ("scratch", "scratch")):
        setattr(g, f, d[k].data_ptr())
    return g, d


@pytest.fixture(params=[1, 0], ids=["bf16-state", "fp32-state"])
def state_mode(request, lmx):
    # the reference's bf16 states between blocks (default) and fp32 states,
    # set alike on the library and the oracle
    lmx.call("lmx_set_gdn_state_bf16", request.param)
    O.lib().orc_set_gdn_state_bf16(request.param)
    yield request.param
    lmx.call("lmx_set_gdn_state_bf16", 1)
    O.lib().orc_set_gdn_state_bf16(1)


@pytest.mark.parametrize("B,T,Hk,Hv", [(2, 3, 2, 4), (4, 3, 16, 32), (3, 1, 1, 2)])
def test_gdn_verify_and_commit_bit_exact(lmx, cuda, state_mode, B, T, Hk, Hv):
    # (4, 3, 16, 32): configuration 4's GDN layer (batch 4, 3 verify tokens,
    # 16 key / 32 value heads of 128)
    c = H.gdn_case(B * 10 + Hv, B=B, T=T, Hk=Hk, Hv=Hv)
    g, d = gdn_device(lmx, cuda, c)
    lmx.call("lmx_gdn_verify", C.byref(g), None)
    cuda.cuda.synchronize()
    ref_out, ref_snap = H.oracle_gdn(c)
    np.testing.assert_array_equal(host(d["out"], np.uint16), ref_out)
    np.testing.assert_array_equal(host(d["snap"], np.float32), ref_snap)
    # state and conv state untouched by verify
    np.testing.assert_array_equal(host(d["state"], np.float32), c["state"])
    # commit (rollback to the accepted prefix), then verify again from there
    acc = np.array([(b * 2) % T for b in range(B)], np.int32)
    dacc = dev(cuda, acc)
    lmx.call("lmx_gdn_commit", C.byref(g), dacc.data_ptr(), None)
    cuda.cuda.synchronize()
    st, conv = H.oracle_commit(c, ref_snap, acc)
    np.testing.assert_array_equal(host(d["state"], np.float32), st)
    np.testing.assert_array_equal(host(d["conv_state"], np.uint16), conv)
    c2 = dict(c, state=st, conv_state=conv, qkv=np.roll(c["qkv"], 1, axis=1))
    d["qkv"].copy_(dev(cuda, c2["qkv"]))
    lmx.call("lmx_gdn_verify", C.byref(g), None)
    cuda.cuda.synchronize()
    out2, snap2 = H.oracle_gdn(c2)
    np.testing.assert_array_equal(host(d["out"], np.uint16), out2)
    np.testing.assert_array_equal(host(d["snap"], np.float32), snap2)


@pytest.mark.parametrize("rows,E,k", [(12, 512, 10), (3, 64, 1), (5, 96, 16)])
def test_moe_route_bit_exact(lmx, cuda, rows, E, k):
    logits = H.moe_route_case(rows + E, rows, E)
    ref_idx, ref_w = H.oracle_route(logits, k)
    dl = dev(cuda, logits)
    idx = cuda.zeros((rows, k), dtype=cuda.int32, device="cuda")
    w = cuda.zeros((rows, k), dtype=cuda.float32, device="cuda")
    lmx.call("lmx_moe_route", dl.data_ptr(), rows, E, k, idx.data_ptr(), w.data_ptr(), None)
    cuda.cuda.synchronize()
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(w.cpu().numpy(), ref_w)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,H_,I,E,k", [(5, 512, 512, 16, 4), (12, 2048, 512, 64, 10)])
def test_moe_experts_bit_exact(lmx, cuda, bits, M, H_, I, E, k):
    # (12, 2048, 512, 64, 10): configuration 4's verify block (4 sequences x
    # 3 tokens, hidden 2048, expert FFN 512, top-10) over 64 of its experts
    c = H.moe_experts_case(M * 3 + bits, M=M, H=H_, I=I, E=E, k=k, bits=bits)
    ref = H.oracle_experts(c)
    keep = []

    def qw(t3):
        ts = [dev(cuda, a) for a in t3]
        keep.extend(ts)
        return lmx.QWeights(w=ts[0].data_ptr(), scales=ts[1].data_ptr(), biases=ts[2].data_ptr())

    gq, uq, dq = qw(c["gate"]), qw(c["up"]), qw(c["down"])
    x, idx, w = dev(cuda, c["x"]), dev(cuda, c["idx"]), dev(cuda, c["w"])
    act = cuda.zeros((M, k, I), dtype=cuda.int16, device="cuda")
    y = cuda.zeros((M, H_), dtype=cuda.int16, device="cuda")
    for _ in range(2):
        lmx.call("lmx_moe_experts", x.data_ptr(), M, H_, I, E, k, idx.data_ptr(), w.data_ptr(), C.byref(gq),
                 C.byref(uq), C.byref(dq), bits, act.data_ptr(), y.data_ptr(), None)
        cuda.cuda.synchronize()
        np.testing.assert_array_equal(host(y, np.uint16), ref)
