"""tcgen05 swap-AB GEMM (through the yk_testing.h hook) against float64 numpy on the
same bf16 operands: tails in every dimension, stream-K cuts at odd places, cluster
split-K, multi-token-tile paths, and run-to-run determinism."""
import numpy as np
import pytest

from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu

SHAPES = [
    # n_out, K, m_tok, grid (0 = production heuristic, > 0 = forced stream-K CTA count,
    #                        < 0 = forced cluster split-K with -grid CTAs per tile)
    (128, 64, 16, 1),
    (256, 128, 16, 1),
    (384, 512, 40, 2),       # 3 tiles x 8 k-blocks over 2 CTAs: the middle tile is cut
    (1000, 320, 7, 5),       # row tail (1000 = 7*128 + 104), token tail, cuts at odd k-blocks
    (256, 200, 33, 1),       # K tail inside a 64-wide k-block (TMA zero fill)
    (512, 1024, 192, 3),     # 4 tiles x 16 k-blocks over 3 CTAs: cut tiles, 2-way fix-up
    (512, 1024, 192, 37),    # each tile cut across ~9 CTAs
    (512, 1024, 192, -3),    # cluster mode: 3-CTA clusters, 32 KB column shares exchanged by copy engine
    (1000, 320, 7, -5),      # cluster mode, one k-block per CTA, row and token tails
    (384, 512, 40, -8),      # cluster mode, 8-CTA clusters
    (256, 200, 33, -4),      # cluster mode with a K tail
    (6144, 4096, 192, 0),    # verify QKV shape (heuristic: cluster mode)
    (4096, 14336, 32, 0),    # down-proj shape at draft batch (cluster mode)
    (512, 256, 300, 0),      # two token tiles (BN = 256)
    (512, 512, 256, -4),     # cluster mode, BN = 256: no room for receive slots, shares loaded over DSMEM
    (28672, 4096, 192, 0),   # verify gate/up: 235 MB of weights (> L2), stream-K; the profiling case
]


@pytest.mark.parametrize("n_out,K,m_tok,grid", SHAPES)
def test_tc_gemm_matches_fp64(engine, n_out, K, m_tok, grid):
    rng = np.random.default_rng(n_out * 7 + K + m_tok)
    W = abi.bf16_bits(rng.normal(0, 0.05, (n_out, K)))
    X = abi.bf16_bits(rng.normal(0, 1.0, (m_tok, K)))
    Y = abi.gemm_bf16_test(engine, W, X, grid)
    Wf = abi.bf16_value(W).astype(np.float64)
    Xf = abi.bf16_value(X).astype(np.float64)
    ref = Xf @ Wf.T
    scale = np.sqrt((Xf ** 2) @ (Wf ** 2).T) + 1e-6  # per-element magnitude of the dot product
    err = np.abs(Y - ref) / scale
    assert np.isfinite(Y).all()
    assert err.max() < 1e-4, f"max scaled error {err.max():.3e}"


def test_tc_gemm_is_deterministic(engine):
    rng = np.random.default_rng(5)
    W = abi.bf16_bits(rng.normal(0, 0.05, (768, 2048)))
    X = abi.bf16_bits(rng.normal(0, 1.0, (96, 2048)))
    a = abi.gemm_bf16_test(engine, W, X, 7)
    b = abi.gemm_bf16_test(engine, W, X, 7)
    c = abi.gemm_bf16_test(engine, W, X, -6)
    d = abi.gemm_bf16_test(engine, W, X, -6)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(c, d)
