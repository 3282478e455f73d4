"""lmx_sdpa_decode_noalloc: the attention entry point for callers that cannot
allocate device memory (it uses a built-in device array instead of caller
scratch).  Its output must equal lmx_sdpa_decode's (bit-exact, the tolerance
the attention tests use) on two calls in a row, which also checks that the
shared array is left ready for the next call.  This file is collected last."""
import ctypes as C
import math

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

D = 128


def _dev(cuda, a):
    view = {np.uint16: np.int16, np.uint32: np.int32}.get(a.dtype.type, None)
    return cuda.from_numpy(np.ascontiguousarray(a.view(view) if view else a)).cuda()


# (bits, T, Hq, cap, exact): the first three in exact mode take the CUDA-core
# kernel; the last two in tensor-core mode the tensor-core kernel -- 40 rows
# per KV head (8 q heads per KV head x 5 verify tokens), and a single-token
# decode over a cache of more than 2048 rows.
@pytest.mark.parametrize("bits,T,Hq,cap,exact", [(16, 5, 16, 300, 1), (8, 1, 16, 300, 1), (4, 6, 16, 300, 1),
                                                 (8, 5, 64, 300, 0), (4, 1, 16, 2304, 0)])
def test_noalloc_matches_caller_scratch_entry(lmx, cuda, mma_threshold, bits, T, Hq, cap, exact):
    mma_threshold(0 if exact else 16)
    rng = np.random.RandomState(7 + bits + T)
    B, Hk = 2, 8
    lens = np.array([17, cap - T], np.int32)
    desc = lmx.KvDesc(batch=B, kv_heads=Hk, head_dim=D, capacity=cap, bits=bits)
    keep = []
    if bits == 16:
        k = _dev(cuda, O.gen_normal_bf16(1, 1, 1.0, B * Hk * cap * D))
        v = _dev(cuda, O.gen_normal_bf16(1, 2, 1.0, B * Hk * cap * D))
        desc.k, desc.v = k.data_ptr(), v.data_ptr()
        keep += [k, v]
    else:
        words = B * Hk * cap * D * bits // 32
        tens = [_dev(cuda, rng.randint(0, 2**32, words, dtype=np.uint64).astype(np.uint32)) for _ in range(2)]
        sb = [_dev(cuda, O.f32_to_bf16(rng.uniform(0.001, 0.05, B * Hk * cap * 2).astype(np.float32)))
              for _ in range(4)]
        desc.k_packed, desc.v_packed = tens[0].data_ptr(), tens[1].data_ptr()
        desc.k_scales, desc.k_biases, desc.v_scales, desc.v_biases = [t.data_ptr() for t in sb]
        keep += tens + sb
    dlen = _dev(cuda, lens)
    desc.lengths = dlen.data_ptr()
    q = _dev(cuda, O.gen_normal_bf16(3, 3, 1.0, B * T * Hq * D))
    scale = float(np.float32(1.0 / math.sqrt(D)))
    nbytes = lmx.lib().lmx_sdpa_scratch_bytes(B, T, Hq, Hk, cap)
    scratch = cuda.zeros(nbytes, dtype=cuda.uint8, device="cuda")
    ref = cuda.empty(B * T * Hq * D, dtype=cuda.int16, device="cuda")
    lmx.call("lmx_sdpa_decode", q.data_ptr(), C.byref(desc), T, Hq, scale, scratch.data_ptr(), nbytes,
             ref.data_ptr(), None)
    for _ in range(2):
        out = cuda.full((B * T * Hq * D,), 7, dtype=cuda.int16, device="cuda")
        lmx.call("lmx_sdpa_decode_noalloc", q.data_ptr(), C.byref(desc), T, Hq, scale, out.data_ptr(), None)
        cuda.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), ref.cpu().numpy())


def test_noalloc_rejects_shapes_beyond_its_array(lmx, cuda):
    B, Hq, Hk, cap, T = 16, 64, 8, 8192, 5
    assert lmx.lib().lmx_sdpa_scratch_bytes(B, T, Hq, Hk, cap) > 16 << 20
    dlen = cuda.zeros(B, dtype=cuda.int32, device="cuda")
    buf = cuda.zeros(16, dtype=cuda.int16, device="cuda")
    desc = lmx.KvDesc(batch=B, kv_heads=Hk, head_dim=D, capacity=cap, bits=16, k=buf.data_ptr(),
                      v=buf.data_ptr(), lengths=dlen.data_ptr())
    rc = lmx.lib().lmx_sdpa_decode_noalloc(buf.data_ptr(), C.byref(desc), T, Hq, 0.088, buf.data_ptr(), None)
    assert rc == 5 and b"16777216" in lmx.lib().lmx_last_error()
