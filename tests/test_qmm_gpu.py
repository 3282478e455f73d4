"""K1 quantized GEMV, RMSNorm and argmax on the B200 vs the CPU oracle.

The CUDA-core paths follow the oracle's canonical fp32 order, so the bar is
bit-exact equality of the bf16 outputs."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def canonical(mma_threshold):
    # every M on the CUDA-core GEMV (the tcgen05 path has its own tests)
    mma_threshold(0)


def dev(torch, a):
    t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else
                         (a.view(np.int32) if a.dtype == np.uint32 else a))
    return t.cuda()


def host_u16(t):
    return t.cpu().numpy().view(np.uint16)


def ptr(t):
    return t.data_ptr()


def run_qmm(lmx, torch, x, wq, s, b, bits, N, K):
    M = x.shape[0]
    dx, dw, ds, db = dev(torch, x), dev(torch, wq), dev(torch, s), dev(torch, b)
    dy = torch.empty((M, N), dtype=torch.int16, device="cuda")
    lmx.call("lmx_quantized_matmul", ptr(dx), ptr(dw), ptr(ds), ptr(db), ptr(dy), M, N, K, 64, bits,
             None)
    torch.cuda.synchronize()
    code = __import__("ctypes").c_uint(0)
    lmx.call("lmx_device_error", __import__("ctypes").byref(code), 1)
    assert code.value == 0
    return host_u16(dy)


SHAPES = [(256, 512), (1000, 1024), (4096, 1024), (1024, 2048), (3072, 1024), (1024, 3072),
          (4096, 4096), (520, 4160), (4096, 12288), (512, 14336)]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 11, 20])
@pytest.mark.parametrize("N,K", SHAPES)
def test_qmm_bit_exact(lmx, cuda, bits, M, N, K):
    wq, s, b = O.gen_sweep_weights(11 + N, 7 + K, N, K, bits)
    x = O.gen_normal_bf16(3 + M, K, 1.0, M * K).reshape(M, K)
    ref = O.qmm(x, wq, s, b, bits)
    got = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    mism = np.argwhere(got != ref)
    assert mism.size == 0, f"{len(mism)} mismatches, first {mism[:3].tolist()}"


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_config2_shapes_bit_exact(lmx, cuda, bits):
    # the op-level sweep's (N, K) set at M in {1, 5}
    for N, K in [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]:
        wq, s, b = O.gen_sweep_weights(2026, 1, N, K, bits)
        for M in (1, 5):
            x = O.gen_normal_bf16(9, M, 1.0, M * K).reshape(M, K)
            np.testing.assert_array_equal(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K),
                                          O.qmm(x, wq, s, b, bits))


@pytest.mark.parametrize("rows,dim", [(1, 1024), (5, 1024), (40, 128), (7, 4096), (300, 8192)])
def test_rms_norm_bit_exact(lmx, cuda, rows, dim):
    x = O.gen_normal_bf16(4, rows, 2.0, rows * dim).reshape(rows, dim)
    w = O.gen_normal_bf16(5, dim, 0.3, dim)
    ref = O.rms_norm(x, w, 1e-6)
    dx, dw = dev(cuda, x), dev(cuda, w)
    dy = cuda.empty_like(dx)
    lmx.call("lmx_rms_norm", ptr(dx), ptr(dw), ptr(dy), rows, dim, 1e-6, None)
    np.testing.assert_array_equal(host_u16(dy), ref)


@pytest.mark.parametrize("rows,V", [(1, 151936), (5, 151936), (3, 1000), (2, 128256)])
def test_argmax_matches(lmx, cuda, rows, V):
    l = O.gen_normal_bf16(6, V, 1.0, rows * V).reshape(rows, V)
    l[0, V // 3] = O.f32_to_bf16(np.float32(30.0))
    l[0, V // 2] = O.f32_to_bf16(np.float32(30.0))  # tie: first index wins
    dl = dev(cuda, l)
    out = cuda.empty(rows, dtype=cuda.int32, device="cuda")
    lmx.call("lmx_argmax", ptr(dl), rows, V, ptr(out), None)
    np.testing.assert_array_equal(out.cpu().numpy(), O.argmax(l))
    assert out[0].item() == V // 3
