"""K1 tensor-core path (tcgen05, M >= 16) on the B200 vs the CPU oracle.

The oracle's path for M >= 16 dequantizes each weight to bf16(fma(s, q, b))
and forms the dot product in double; the device accumulates the same bf16
products in fp32 on the tensor cores in the hardware's order.  The bar per
output: |got - ref| <= one bf16 ulp of ref (the two sides round nearly equal
fp32 values, which may straddle a rounding boundary) plus 2^-16 *
sum_k |w_k x_k| (a bound on fp32 accumulation error far above its typical
size)."""
import numpy as np
import pytest

import oracle_lib as O
from test_qmm_gpu import run_qmm

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def tcgen05_for_every_m(lmx):
    # the mid-batch mma.sync GEMM (test_qmm_tcs_gpu) off on both sides: every
    # M at or above the threshold takes tcgen05
    lmx.call("lmx_set_gemm_tcs_max_m", 0)
    O.lib().orc_set_tcs_max_m(0)
    yield
    lmx.call("lmx_set_gemm_tcs_max_m", 0)
    O.lib().orc_set_tcs_max_m(0)


def dequant_f32(wq, s, b, N, K, bits):
    return O.bf16_to_f32(O.dequantize(wq, s, b, K, 64, bits)).reshape(N, K).astype(np.float64)


def check_close(got, ref, x, wd):
    g = O.bf16_to_f32(got).astype(np.float64)
    r = O.bf16_to_f32(ref).astype(np.float64)
    xf = O.bf16_to_f32(x).astype(np.float64)
    S = np.abs(xf) @ np.abs(wd).T
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(r), 1e-30))) - 7)
    tol = ulp + S * 2.0 ** -16 + 1e-30
    err = np.abs(g - r)
    bad = np.argwhere(err > tol)
    assert bad.size == 0, (f"{len(bad)} outputs out of tolerance, first {bad[:3].tolist()}, "
                           f"worst ratio {float((err / tol).max()):.3g}")
    return float((got == ref).mean())


SHAPES = [(256, 512), (1000, 1024), (4096, 1024), (3072, 1024), (1024, 3072), (520, 4160),
          (4096, 4096)]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [16, 17, 48, 100, 256, 300])
@pytest.mark.parametrize("N,K", SHAPES)
def test_qmm_mma_within_tolerance(lmx, cuda, mma_threshold, bits, M, N, K):
    mma_threshold(16)
    wq, s, b = O.gen_sweep_weights(11 + N, 7 + K, N, K, bits)
    x = O.gen_normal_bf16(3 + M, K, 1.0, M * K).reshape(M, K)
    ref = O.qmm(x, wq, s, b, bits)
    got = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    exact = check_close(got, ref, x, dequant_f32(wq, s, b, N, K, bits))
    assert exact > 0.9, f"only {exact:.3f} of outputs equal the double-accumulated result"


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_mma_config2_shapes(lmx, cuda, mma_threshold, bits):
    # the op-level sweep's (N, K) set at M in {16, 32}
    mma_threshold(16)
    for N, K in [(4096, 4096), (14336, 4096), (4096, 14336)]:
        wq, s, b = O.gen_sweep_weights(2026, 1, N, K, bits)
        wd = dequant_f32(wq, s, b, N, K, bits)
        for M in (16, 32):
            x = O.gen_normal_bf16(9, M, 1.0, M * K).reshape(M, K)
            check_close(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K), O.qmm(x, wq, s, b, bits), x, wd)


def test_qmm_mma_agrees_with_canonical_order(lmx, cuda, mma_threshold):
    # the two device paths on the same inputs: within the bf16 rounding of
    # each other (they differ by the dequantized weight's rounding and the
    # summation order)
    N, K, M, bits = 2048, 4096, 32, 4
    wq, s, b = O.gen_sweep_weights(5, 6, N, K, bits)
    x = O.gen_normal_bf16(8, M, 1.0, M * K).reshape(M, K)
    mma_threshold(16)
    a = O.bf16_to_f32(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)).astype(np.float64)
    mma_threshold(0)
    c = O.bf16_to_f32(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)).astype(np.float64)
    rms = np.sqrt((c ** 2).mean())
    assert np.abs(a - c).max() <= 2e-2 * rms
