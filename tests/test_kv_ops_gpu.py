"""KV-cache ops through the C ABI over an engine cache: lmx_cache_kv (the
layer as an lmx_kv view), lmx_kv_append (the reference's update: rows at
each sequence's length, quantized on append, lengths advanced), and
lmx_kv_set_position (rollback) -- bit-exact against the oracle's quantizer;
a block past the capacity is refused with device error 0x42."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

D = 128
CFG = dict(hidden=512, layers=2, inter=1024, heads=4, kv_heads=2, head_dim=128, vocab=1000,
           rope_theta=1e6, eps=1e-6, qk_norm=1, tied=1, bits=4, group_size=64)


def d2h(dst, src_addr, nbytes):
    # the CUDA runtime the library itself loaded (cudaMemcpyDeviceToHost = 2)
    rt = C.CDLL("libcudart.so.12")
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    assert rt.cudaMemcpy(dst.ctypes.data, C.c_void_p(src_addr), nbytes, 2) == 0


def rows_of(kv, which, b, h, r0, n):
    """Rows [r0, r0+n) of (sequence b, KV head h): bf16 values, or (codes,
    scales, biases) for a quantized cache, copied from the device."""
    row0 = (b * kv.kv_heads + h) * kv.capacity + r0
    if kv.bits == 16:
        out = np.zeros((n, D), np.uint16)
        d2h(out, (kv.k if which == "k" else kv.v) + row0 * D * 2, out.nbytes)
        return out
    wpr = D * kv.bits // 32
    w = np.zeros((n, wpr), np.uint32)
    s = np.zeros((n, 2), np.uint16)
    bb = np.zeros((n, 2), np.uint16)
    d2h(w, (kv.k_packed if which == "k" else kv.v_packed) + row0 * wpr * 4, w.nbytes)
    d2h(s, (kv.k_scales if which == "k" else kv.v_scales) + row0 * 4, s.nbytes)
    d2h(bb, (kv.k_biases if which == "k" else kv.v_biases) + row0 * 4, bb.nbytes)
    return w, s, bb


@pytest.mark.parametrize("bits", [16, 8, 4])
def test_kv_append_and_set_position(lmx, cuda, bits):
    g = lmx.Model(CFG, 5)
    B, Hk, cap, T = 2, CFG["kv_heads"], 40, 7
    c = C.c_void_p()
    lmx.call("lmx_cache_create", g.h, CFG["layers"], B, cap, bits, 8, C.byref(c))
    kv = lmx.KvDesc()
    lmx.call("lmx_cache_kv", c, 1, C.byref(kv))
    assert kv.bits == bits and kv.batch == B and kv.kv_heads == Hk and kv.capacity >= cap
    rng = np.random.RandomState(bits)
    code = C.c_uint(0)
    lmx.call("lmx_device_error", C.byref(code), 1)
    blocks = []
    for i in range(2):
        kn = O.gen_normal_bf16(rng.randint(1 << 30), 1, 1.0, B * Hk * T * D).reshape(B, Hk, T, D)
        vn = O.gen_normal_bf16(rng.randint(1 << 30), 2, 1.0, B * Hk * T * D).reshape(B, Hk, T, D)
        dk = cuda.from_numpy(kn.view(np.int16).copy()).cuda()
        dv = cuda.from_numpy(vn.view(np.int16).copy()).cuda()
        lmx.call("lmx_kv_append", C.byref(kv), dk.data_ptr(), dv.data_ptr(), T, None)
        cuda.cuda.synchronize()
        blocks.append((kn, vn))
        if i == 0:  # roll sequence 1 back by 3 rows: the next block overwrites them
            lmx.call("lmx_kv_set_position", C.byref(kv), 1, T - 3, None)
    lens = np.zeros(B, np.int32)
    for b in range(B):
        n = C.c_int()
        lmx.call("lmx_cache_len", c, b, C.byref(n))
        lens[b] = n.value
    assert list(lens) == [2 * T, 2 * T - 3]
    for b in range(B):
        for h in range(Hk):
            # sequence 1 was rolled back by 3 rows: the second block
            # overwrote the first block's last 3 rows
            starts = [0, T if b == 0 else T - 3]
            counts = [T if b == 0 else T - 3, T]
            for (kn, vn), r0, cnt in zip(blocks, starts, counts):
                for which, src in (("k", kn), ("v", vn)):
                    got = rows_of(kv, which, b, h, r0, cnt)
                    x = np.ascontiguousarray(src[b, h, :cnt])
                    if bits == 16:
                        np.testing.assert_array_equal(got, x)
                    else:
                        wq, s, bb = O.quantize(x, 64, bits)
                        np.testing.assert_array_equal(got[0], wq)
                        np.testing.assert_array_equal(got[1], s)
                        np.testing.assert_array_equal(got[2], bb)
    lmx.call("lmx_device_error", C.byref(code), 1)
    assert code.value == 0
    # past the capacity: refused, lengths unchanged, device error 0x42
    big = kv.capacity - int(lens.min()) + 1
    z = cuda.zeros(B * Hk * big * D, dtype=cuda.int16, device="cuda")
    lmx.call("lmx_kv_append", C.byref(kv), z.data_ptr(), z.data_ptr(), big, None)
    cuda.cuda.synchronize()
    lmx.call("lmx_device_error", C.byref(code), 1)
    assert code.value == 0x42
    n = C.c_int()
    lmx.call("lmx_cache_len", c, 1, C.byref(n))
    assert n.value == lens[1]
    lmx.call("lmx_cache_free", c)
    g.close()
