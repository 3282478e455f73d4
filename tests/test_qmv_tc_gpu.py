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


@pytest.fixture
def rows_tiles(lmx):
    def set_(t):
        lmx.call("lmx_set_gemv_tc_rows_min_tiles", t)

    yield set_
    set_(1024)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [4, 8, 13])
@pytest.mark.parametrize("N,K", [(1000, 1024), (4096, 4096), (520, 4160), (20000, 1024)])
def test_qmv_tc_rows_within_tolerance(lmx, cuda, mma_threshold, gemv_tc, rows_tiles, bits, M, N, K):
    # the warp-per-tile form (forced for every matrix here; by default for
    # >= 1024 tiles, e.g. the 20000-row case): same bound as the split form
    mma_threshold(16)
    gemv_tc(4)
    rows_tiles(1)
    wq, s, b = O.gen_sweep_weights(21 + N, 5 + K, N, K, bits)
    x = O.gen_normal_bf16(9 + M, K, 1.0, M * K).reshape(M, K)
    got = run_qmm(lmx, cuda, x, wq, s, b, bits, N, K)
    exact = check_close(got, O.qmm(x, wq, s, b, bits), x, magnitudes(wq, s, b, N, K, bits))
    assert exact > 0.9, f"only {exact:.3f} of outputs equal the canonical GEMV's"


def test_qmv_tc_rows_in_the_decoder(lmx, cuda, mma_threshold, gemv_tc, rows_tiles):
    # every PLAIN / RESID GEMV of a decoder through the warp-per-tile form
    # (q|k|v and the lm_head with the fused RMSNorm, o_proj / down_proj with
    # the residual add): logits within the engine's tensor-core tolerance of
    # the oracle, and of the split form
    import ctypes as C
    from test_engine_gpu import TINY, assert_logits_close, oracle_cfg
    mma_threshold(16)
    gemv_tc(4)
    cfg = dict(TINY, tied=0)
    g = lmx.Model(cfg, 99)
    o = O.lib().orc_model_create(C.byref(oracle_cfg(cfg)), 99)
    L, V, B = cfg["layers"], cfg["vocab"], 4
    rng = np.random.RandomState(3)
    pre = rng.randint(0, V, (B, 12)).astype(np.int32)
    outs = []
    try:
        for t in (1, 1024):
            rows_tiles(t)
            gc = C.c_void_p()
            lmx.call("lmx_cache_create", g.h, L, B, 64, 16, 12, C.byref(gc))
            oc = O.lib().orc_cache_create(o, L, B, 64, 16)
            for T in (3, 1, 2):  # M = 12, 4, 8: every block on the small-batch GEMV
                tok = pre[:, :T].copy()
                gl = np.zeros((B, T, V), np.uint16)
                ol = np.zeros((B, T, V), np.uint16)
                lmx.call("lmx_forward", g.h, gc, L, tok.ctypes.data, B, T, gl.ctypes.data)
                assert O.lib().orc_forward(o, oc, L, O.ptr(tok), B, T, O.ptr(ol)) == 0
                assert_logits_close(gl, ol, f"rows_min_tiles {t}, T={T}")
                outs.append(gl)
            lmx.call("lmx_cache_free", gc)
            O.lib().orc_cache_free(oc)
        for a, b in zip(outs[:3], outs[3:]):
            assert_logits_close(a, b, "warp-per-tile vs split form")
    finally:
        g.close()
        O.lib().orc_model_free(o)
    assert lmx.lib().lmx_set_gemv_tc_rows_min_tiles(-1) != 0
