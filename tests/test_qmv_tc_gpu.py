"""K1 small-batch tensor-core GEMV (mma.sync, 4 <= M <= 16 below the tcgen05
threshold) on the B200 vs the CPU oracle.

The path keeps MLX qmv's math (per 64-k group s * sum q x + b * sum x, the
codes exact on the tensor cores), so the oracle's canonical GEMV is the
reference; only the fp32 summation order differs.  The bar per output: one
bf16 ulp of the reference plus 2^-16 * sum_k (s q_k + |b|) |x_k| (the
magnitudes the two fp32 sums run over; far above the typical error).  The
fused epilogues (residual add, SwiGLU) and the split-K clusters run inside
the decoder and are covered by the engine tests' tensor-core cases."""
import numpy as np
import pytest

import oracle_lib as O
from test_qmm_gpu import run_qmm

pytestmark = pytest.mark.gpu

# split-K clusters of 1 (256x512, 1000x1024, ...), 2 (1024x3072) and 4
# (520x4160, 512x14336) CTAs
SHAPES = [(256, 512), (1000, 1024), (4096, 1024), (3072, 1024), (1024, 3072), (520, 4160),
          (4096, 4096), (512, 14336)]


@pytest.fixture
def gemv_tc(lmx):
    def set_(m):
        lmx.call("lmx_set_gemv_tc_min_m", m)

    yield set_
    set_(4)


def magnitudes(wq, s, b, N, K, bits):
    """(s q + |b|) per weight, float64 [N, K]."""
    per = 32 // bits
    codes = np.zeros((N, K), np.float64)
    w = wq.reshape(N, K // per)
    for j in range(per):
        codes[:, j::per] = (w >> np.uint32(j * bits)) & np.uint32(2**bits - 1)
    sc = np.repeat(O.bf16_to_f32(s).reshape(N, -1).astype(np.float64), 64, 1)
    bi = np.repeat(np.abs(O.bf16_to_f32(b).reshape(N, -1).astype(np.float64)), 64, 1)
    return codes * sc + bi


def check_close(got, ref, x, mag):
    g = O.bf16_to_f32(got).astype(np.float64)
    r = O.bf16_to_f32(ref).astype(np.float64)
    S = np.abs(O.bf16_to_f32(x).astype(np.float64)) @ mag.T
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(r), 1e-30))) - 7)
    tol = ulp + S * 2.0 ** -16 + 1e-30
    err = np.abs(g - r)
    bad = np.argwhere(err > tol)
    assert bad.size == 0, (f"{len(bad)} outputs out of tolerance, first {bad[:3].tolist()}, "
                           f"worst ratio {float((err / tol).max()):.3g}")
    return float((got == ref).mean())


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [4, 5, 8, 9, 12, 15])
@pytest.mark.parametrize("N,K", SHAPES)
def test_qmv_tc_within_tolerance(lmx, cuda, mma_threshold, gemv_tc, bits, M, N, K):
    mma_threshold(16)
    gemv_tc(4)
    wq, s, b = O.gen_sweep_weights(11 + N, 7 + K, N, K, bits)
    x = O.gen_normal_bf16(3 + M, K, 1.0, M * K).reshape(M, K)
    ref = O.qmm(x, wq, s, b, bits)
    got = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    exact = check_close(got, ref, x, magnitudes(wq, s, b, N, K, bits))
    assert exact > 0.9, f"only {exact:.3f} of outputs equal the canonical GEMV's"


@pytest.mark.parametrize("bits", [4, 8])
def test_qmv_tc_sixteen_rows_below_a_higher_threshold(lmx, cuda, mma_threshold, gemv_tc, bits):
    # with the tcgen05 threshold above 16, M = 16 takes this path (two
    # 8-token column tiles full) and M = 20 the canonical GEMV
    mma_threshold(32)
    gemv_tc(4)
    N, K = 1000, 2048
    wq, s, b = O.gen_sweep_weights(3, 4, N, K, bits)
    mag = magnitudes(wq, s, b, N, K, bits)
    x = O.gen_normal_bf16(12, 16, 1.0, 16 * K).reshape(16, K)
    check_close(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K), O.qmm(x, wq, s, b, bits), x, mag)
    x = O.gen_normal_bf16(13, 20, 1.0, 20 * K).reshape(20, K)
    got, ref = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K), O.qmm(x, wq, s, b, bits)
    np.testing.assert_array_equal(got, ref)


def test_qmv_tc_off_restores_canonical_order(lmx, cuda, mma_threshold, gemv_tc):
    # threshold 0: M < 16 back on the canonical GEMV, bit-exact
    mma_threshold(16)
    gemv_tc(0)
    N, K, bits = 1024, 2048, 4
    wq, s, b = O.gen_sweep_weights(5, 6, N, K, bits)
    for M in (4, 12):
        x = O.gen_normal_bf16(8 + M, M, 1.0, M * K).reshape(M, K)
        np.testing.assert_array_equal(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K), O.qmm(x, wq, s, b, bits))


def test_gemv_tc_threshold_validation(lmx, gemv_tc):
    assert lmx.lib().lmx_set_gemv_tc_min_m(17) != 0
    assert lmx.lib().lmx_set_gemv_tc_min_m(-1) != 0
    gemv_tc(6)
    assert lmx.lib().lmx_gemv_tc_min_m() == 6
