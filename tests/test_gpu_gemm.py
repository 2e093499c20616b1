"""tcgen05 swap-AB GEMM (through the yk_testing.h hook) against float64 numpy on the
same bf16 operands: tails in every dimension, split-K and multi-token-tile paths."""
import numpy as np
import pytest

from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu

SHAPES = [
    # n_out, K, m_tok, forced splits (0 = heuristic)
    (128, 64, 16, 1),
    (256, 128, 16, 1),
    (384, 512, 40, 1),
    (1000, 320, 7, 1),       # row tail (1000 = 7*128 + 104), k tail none, token tail
    (256, 200, 33, 1),       # K tail inside a 64-wide k-block (TMA zero fill)
    (512, 1024, 192, 4),     # split-K with last-arriver fixup
    (6144, 4096, 192, 0),    # verify QKV shape, heuristic split
    (4096, 14336, 32, 0),    # down-proj shape at draft batch
    (512, 256, 300, 1),      # two token tiles (BN = 256)
    (28672, 4096, 192, 0),   # verify gate/up shape: 235 MB of weights (> L2), the profiling case
]


@pytest.mark.parametrize("n_out,K,m_tok,splits", SHAPES)
def test_tc_gemm_matches_fp64(engine, n_out, K, m_tok, splits):
    rng = np.random.default_rng(n_out * 7 + K + m_tok)
    W = abi.bf16_bits(rng.normal(0, 0.05, (n_out, K)))
    X = abi.bf16_bits(rng.normal(0, 1.0, (m_tok, K)))
    Y = abi.gemm_bf16_test(engine, W, X, splits)
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
    a = abi.gemm_bf16_test(engine, W, X, 6)
    b = abi.gemm_bf16_test(engine, W, X, 6)
    np.testing.assert_array_equal(a, b)
