"""The bounded wait of the tensor-parallel all-reduce runs out on one GPU.

A size-2 communicator whose peer block is a zeroed buffer in this GPU's own
memory (attached by pointer): the peer's arrival flag is never written, so
the kernel's wait must give up after its 2 s limit, set the device error
word to 0x71 and return with h and xn untouched.  No GPU fault is involved:
the wait is bounded and the kernel returns normally."""
import ctypes as C
import time

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu


def test_allreduce_wait_runs_out_and_reports(lmx, cuda):
    R, H = 4, 1024
    comm = C.c_void_p()
    lmx.call("lmx_tp_comm_create", 0, 2, R, H, C.byref(comm))
    nbytes = lmx.lib().lmx_tp_comm_block_bytes(comm)
    assert nbytes > 2 * R * H * 2
    fake_peer = cuda.zeros(nbytes, dtype=cuda.uint8, device="cuda")  # nothing ever arrives here
    try:
        lmx.call("lmx_tp_comm_attach", comm, 1, fake_peer.data_ptr())
        assert lmx.lib().lmx_tp_comm_attach(comm, 1, fake_peer.data_ptr()) != 0  # already open
        code = C.c_uint(0)
        lmx.call("lmx_device_error", C.byref(code), 1)  # start from a clear error word
        h0 = O.gen_normal_bf16(5, 1, 1.0, R * H)
        h = cuda.from_numpy(h0.view(np.int16).copy()).cuda()
        part = cuda.from_numpy(O.gen_normal_bf16(5, 2, 1.0, R * H).view(np.int16).copy()).cuda()
        w = cuda.ones(H, dtype=cuda.bfloat16, device="cuda")
        xn = cuda.full((R * H,), 7, dtype=cuda.int16, device="cuda")
        cuda.cuda.synchronize()
        t0 = time.perf_counter()
        lmx.call("lmx_tp_allreduce_rmsnorm", comm, part.data_ptr(), R, H, h.data_ptr(), w.data_ptr(),
                 C.c_float(1e-6), xn.data_ptr(), None)
        cuda.cuda.synchronize()
        dt = time.perf_counter() - t0
        lmx.call("lmx_device_error", C.byref(code), 1)
        assert code.value == 0x71, hex(code.value)
        assert 1.9 < dt < 20.0, dt
        np.testing.assert_array_equal(h.cpu().numpy().view(np.uint16), h0)
        assert (xn.cpu().numpy() == 7).all()
    finally:
        lmx.call("lmx_tp_comm_free", comm)


def test_allreduce_single_rank_comm_is_residual_plus_norm(lmx, cuda):
    # size 1: no peers, no wait; h = bf16(h + bf16(partial)), xn = rms_norm(h)
    R, H = 3, 512
    comm = C.c_void_p()
    lmx.call("lmx_tp_comm_create", 0, 1, R, H, C.byref(comm))
    try:
        h0 = O.gen_normal_bf16(6, 1, 1.0, R * H)
        p0 = O.gen_normal_bf16(6, 2, 1.0, R * H)
        w0 = O.gen_normal_bf16(6, 3, 1.0, H)
        dev = lambda a: cuda.from_numpy(a.view(np.int16).copy()).cuda()
        h, part, w = dev(h0), dev(p0), dev(w0)
        xn = cuda.zeros(R * H, dtype=cuda.int16, device="cuda")
        lmx.call("lmx_tp_allreduce_rmsnorm", comm, part.data_ptr(), R, H, h.data_ptr(), w.data_ptr(),
                 C.c_float(1e-6), xn.data_ptr(), None)
        cuda.cuda.synchronize()
        code = C.c_uint(0)
        lmx.call("lmx_device_error", C.byref(code), 0)
        assert code.value == 0
        ref_h = O.f32_to_bf16(O.bf16_to_f32(h0) + O.bf16_to_f32(p0))
        np.testing.assert_array_equal(h.cpu().numpy().view(np.uint16), ref_h)
        ref_x = O.rms_norm(ref_h.reshape(R, H), w0, 1e-6).ravel()
        np.testing.assert_array_equal(xn.cpu().numpy().view(np.uint16), ref_x)
    finally:
        lmx.call("lmx_tp_comm_free", comm)
