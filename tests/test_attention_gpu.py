"""lmx_sdpa_decode (K2) vs the oracle's SDPA over the same cache.  Exact mode
(tensor-core threshold 0): bit-exact for bf16 and for 8/4-bit affine caches
(dequantized the same way on both sides).  Tensor-core mode (blocks of >= 16
query rows per KV head on mma.sync): within a tolerance."""
import ctypes as C
import math

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

D = 128


def make_cache(rng, B, Hk, cap, bits):
    if bits == 16:
        k = O.gen_normal_bf16(rng.randint(1 << 30), 1, 1.0, B * Hk * cap * D).reshape(B, Hk, cap, D)
        v = O.gen_normal_bf16(rng.randint(1 << 30), 2, 1.0, B * Hk * cap * D).reshape(B, Hk, cap, D)
        return dict(k=k, v=v), k, v
    per = 32 // bits
    kq = rng.randint(0, 2**32, (B, Hk, cap, D // per), dtype=np.uint64).astype(np.uint32)
    vq = rng.randint(0, 2**32, (B, Hk, cap, D // per), dtype=np.uint64).astype(np.uint32)
    sc = lambda: O.f32_to_bf16(np.abs(rng.normal(0, 0.2, (B, Hk, cap, 2))).astype(np.float32) / (2**bits - 1))
    ks, vs = sc(), sc()
    kb = O.f32_to_bf16(rng.normal(0, 1, (B, Hk, cap, 2)).astype(np.float32))
    vb = O.f32_to_bf16(rng.normal(0, 1, (B, Hk, cap, 2)).astype(np.float32))
    rows = B * Hk * cap
    kd = O.dequantize(kq.reshape(rows, -1), ks.reshape(rows, 2), kb.reshape(rows, 2), D, 64, bits)
    vd = O.dequantize(vq.reshape(rows, -1), vs.reshape(rows, 2), vb.reshape(rows, 2), D, 64, bits)
    return (dict(kq=kq, vq=vq, ks=ks, kb=kb, vs=vs, vb=vb), kd.reshape(B, Hk, cap, D),
            vd.reshape(B, Hk, cap, D))


def to_dev(cuda, a):
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, None)
    return cuda.from_numpy(np.ascontiguousarray(a.view(view) if view else a)).cuda()


def kv_desc(lmx, dev, B, Hk, cap, bits, lens):
    d = lmx.KvDesc(batch=B, kv_heads=Hk, head_dim=D, capacity=cap, bits=bits)
    if bits == 16:
        d.k, d.v = dev["k"].data_ptr(), dev["v"].data_ptr()
    else:
        d.k_packed, d.v_packed = dev["kq"].data_ptr(), dev["vq"].data_ptr()
        d.k_scales, d.k_biases = dev["ks"].data_ptr(), dev["kb"].data_ptr()
        d.v_scales, d.v_biases = dev["vs"].data_ptr(), dev["vb"].data_ptr()
    d.lengths = lens.data_ptr()
    return d


def oracle_attention(q, kd, vd, lens, T, Hq, Hk, cap, scale):
    B = kd.shape[0]
    out = np.empty((B, T, Hq, D), np.uint16)
    for b in range(B):
        qb = np.ascontiguousarray(q[b])
        o = np.empty(T * Hq * D, np.uint16)
        O.lib().orc_sdpa(O.ptr(qb), O.ptr(np.ascontiguousarray(kd[b])), O.ptr(np.ascontiguousarray(vd[b])),
                         O.ptr(o), T, Hq, Hk, D, cap, int(lens[b]), scale)
        out[b] = o.reshape(T, Hq, D)
    return out


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("T,Hq,Hk,cap", [(1, 16, 8, 420), (5, 16, 8, 420), (6, 32, 8, 420), (40, 4, 2, 420),
                                         (1, 16, 8, 3300), (6, 32, 8, 3300)])
def test_sdpa_decode_bit_exact(lmx, cuda, mma_threshold, bits, T, Hq, Hk, cap):
    # cap 420: 4 splits of 128 keys; cap 3300: 26 splits (long cache, the
    # combine over many partials)
    mma_threshold(0)
    rng = np.random.RandomState(bits * 100 + T)
    B = 3
    lens = np.array([0, 123, cap - T - 1][:B], np.int32)
    host, kd, vd = make_cache(rng, B, Hk, cap, bits)
    dev = {k: to_dev(cuda, v) for k, v in host.items()}
    dlen = to_dev(cuda, lens)
    q = O.gen_normal_bf16(rng.randint(1 << 30), 3, 1.0, B * T * Hq * D).reshape(B, T, Hq, D)
    dq = to_dev(cuda, q)
    out = cuda.empty((B, T, Hq, D), dtype=cuda.int16, device="cuda")
    desc = kv_desc(lmx, dev, B, Hk, cap, bits, dlen)
    nbytes = lmx.lib().lmx_sdpa_scratch_bytes(B, T, Hq, Hk, cap)
    scratch = cuda.zeros(nbytes, dtype=cuda.uint8, device="cuda")
    scale = float(np.float32(1.0 / math.sqrt(D)))
    for _ in range(2):  # the scratch is left ready for the next call
        lmx.call("lmx_sdpa_decode", dq.data_ptr(), C.byref(desc), T, Hq, scale, scratch.data_ptr(), nbytes,
                 out.data_ptr(), None)
        cuda.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        ref = oracle_attention(q, kd, vd, lens, T, Hq, Hk, cap, np.float32(scale))
        bad = np.argwhere(got != ref)
        assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:3].tolist()}"


def test_sdpa_decode_rejects_small_scratch(lmx, cuda):
    B, Hk, cap = 1, 8, 256
    lens = to_dev(cuda, np.zeros(1, np.int32))
    k = cuda.zeros(B * Hk * cap * D, dtype=cuda.int16, device="cuda")
    desc = lmx.KvDesc(batch=B, kv_heads=Hk, head_dim=D, capacity=cap, bits=16, k=k.data_ptr(),
                      v=k.data_ptr(), lengths=lens.data_ptr())
    q = cuda.zeros(16 * D, dtype=cuda.int16, device="cuda")
    rc = lmx.lib().lmx_sdpa_decode(q.data_ptr(), C.byref(desc), 1, 16, 0.088, q.data_ptr(), 16,
                                   q.data_ptr(), None)
    assert rc == 1 and b"scratch" in lmx.lib().lmx_last_error()


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("T,Hq,Hk,cap", [(5, 64, 8, 8300), (6, 32, 8, 1100), (40, 4, 2, 420),
                                         (2, 16, 2, 300), (5, 8, 1, 700), (1, 32, 8, 2100),
                                         (1, 16, 8, 3000), (1, 16, 8, 300)])
def test_sdpa_tensor_core_within_tolerance(lmx, cuda, mma_threshold, bits, T, Hq, Hk, cap):
    # G*T query rows per KV head: 40 (Llama-3-70B verify, 8k cache), 24
    # (Qwen3-8B verify), 80 (two row tiles), 16 (one m16 tile), 40 with a
    # single KV head; and single-token decode (4 and 2 rows) over long and
    # short caches, which in tensor-core mode take the tensor-core kernel
    # too (lmx_set_sdpa_tc_min_cache, default every block).  Tolerance: the
    # products accumulate in the tensor core's order, exponentials come from
    # the hardware ex2 and p keeps ~16 bits -> at most a few bf16 ulps.
    mma_threshold(16)
    rng = np.random.RandomState(bits * 7 + T + Hq)
    B = 3
    lens = np.array([0, 123, cap - T - 1], np.int32)
    host, kd, vd = make_cache(rng, B, Hk, cap, bits)
    dev = {k: to_dev(cuda, v) for k, v in host.items()}
    dlen = to_dev(cuda, lens)
    q = O.gen_normal_bf16(rng.randint(1 << 30), 3, 1.0, B * T * Hq * D).reshape(B, T, Hq, D)
    dq = to_dev(cuda, q)
    out = cuda.empty((B, T, Hq, D), dtype=cuda.int16, device="cuda")
    desc = kv_desc(lmx, dev, B, Hk, cap, bits, dlen)
    nbytes = lmx.lib().lmx_sdpa_scratch_bytes(B, T, Hq, Hk, cap)
    scratch = cuda.zeros(nbytes, dtype=cuda.uint8, device="cuda")
    scale = float(np.float32(1.0 / math.sqrt(D)))
    ref = O.bf16_to_f32(oracle_attention(q, kd, vd, lens, T, Hq, Hk, cap, np.float32(scale)))
    first = None
    for _ in range(2):  # deterministic, and the scratch is left ready
        lmx.call("lmx_sdpa_decode", dq.data_ptr(), C.byref(desc), T, Hq, scale, scratch.data_ptr(), nbytes,
                 out.data_ptr(), None)
        cuda.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16).copy()
        g = O.bf16_to_f32(got)
        tol = 1e-2 + np.abs(ref) * 2.0 ** -7
        bad = np.abs(g - ref) > tol
        assert not bad.any(), f"{int(bad.sum())} out of tolerance, max |diff| {np.abs(g - ref).max():.4g}"
        if first is None:
            first = got
        else:
            np.testing.assert_array_equal(got, first)
