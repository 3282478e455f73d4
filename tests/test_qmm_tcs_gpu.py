"""K1 mid-batch tensor-core GEMM (mma.sync on the exact codes, 16 <= M <= 64
in tensor-core mode) on the B200 vs the CPU oracle's canonical GEMV.

The kernel keeps MLX qmv's math (per 64-k group s * sum q x + b * sum x), so
the canonical GEMV is the reference and the bar is the small-batch GEMV's:
one bf16 ulp plus 2^-16 * sum_k (s q_k + |b|) |x_k| per output.  Shapes
cover split-K clusters of 1 to 8 CTAs, an odd group count (K = 4160), row
counts that are not multiples of 16 or 128, and every token-tile width
(M <= 24, 32, 48, 64).  The fused epilogues (residual add, SwiGLU) run in
the decoder and are covered by the engine's tensor-core tests."""
import numpy as np
import pytest

import oracle_lib as O
from test_qmm_gpu import run_qmm
from test_qmv_tc_gpu import check_close, magnitudes

pytestmark = pytest.mark.gpu

SHAPES = [(256, 512), (1000, 1024), (4096, 1024), (1024, 3072), (520, 4160), (3000, 4096), (6144, 4096)]


@pytest.fixture
def tcs(lmx):
    def set_(m):
        lmx.call("lmx_set_gemm_tcs_max_m", m)
        O.lib().orc_set_tcs_max_m(m)

    yield set_
    set_(0)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [16, 17, 24, 31, 33, 48, 64])
@pytest.mark.parametrize("N,K", SHAPES)
def test_qmm_tcs_within_tolerance(lmx, cuda, mma_threshold, tcs, bits, M, N, K):
    mma_threshold(16)
    tcs(64)
    wq, s, b = O.gen_sweep_weights(31 + N, 9 + K, N, K, bits)
    x = O.gen_normal_bf16(5 + M, K, 1.0, M * K).reshape(M, K)
    ref = O.qmm(x, wq, s, b, bits)  # canonical GEMV: M <= the oracle's bound
    got = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    exact = check_close(got, ref, x, magnitudes(wq, s, b, N, K, bits))
    assert exact > 0.9, f"only {exact:.3f} of outputs equal the canonical GEMV's"


def test_qmm_tcs_deterministic_and_switchable(lmx, cuda, mma_threshold, tcs):
    # run to run identical; off (0) -> M = 48 on tcgen05 again, which agrees
    # within the two paths' tolerances; the bound is validated
    mma_threshold(16)
    N, K, M, bits = 4096, 4096, 48, 4
    wq, s, b = O.gen_sweep_weights(7, 8, N, K, bits)
    x = O.gen_normal_bf16(4, M, 1.0, M * K).reshape(M, K)
    tcs(64)
    a1 = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    a2 = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    np.testing.assert_array_equal(a1, a2)
    tcs(0)
    t = O.bf16_to_f32(run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)).astype(np.float64)
    g = O.bf16_to_f32(a1).astype(np.float64)
    assert np.abs(g - t).max() <= 2e-2 * max(1.0, np.abs(t).max())
    assert lmx.lib().lmx_set_gemm_tcs_max_m(65) != 0
    assert lmx.lib().lmx_set_gemm_tcs_max_m(-1) != 0
