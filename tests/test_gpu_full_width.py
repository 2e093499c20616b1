"""Verify forward at the benchmarked model widths against the bf16-emulating oracle.

The other forward tests run narrow models; these run the real widths of the two
benchmarked targets, with two layers plus the LM head, on a ragged verify batch
over long paged contexts:

* Llama-3-8B shape: d 4096, 32/8 heads x 128, SwiGLU FFN 14336, RoPE theta 5e5,
  vocab 128256; 32 sequences with contexts U[512, 2048], k + 1 = 6 new tokens each.
* Gemma-2-9B shape: d 3584, 16/8 heads x 256, GeGLU FFN 14336, attention cap 50,
  final cap 30, window 4096 on even layers, eps 1e-6, vocab 256000; 16 sequences
  with contexts U[2048, 8192] (both sides of the window), k + 1 = 5 new tokens.

The contexts' K/V pages are synthetic N(0, 1) values (filled on the device, read
back into the oracle's pool), so no prompt has to be pushed through the CPU
oracle; the new tokens' K/V are written by both sides.  Tolerance: max |dlogit|
<= 2e-2 * max|logit| (as the narrow bf16 tests), greedy tokens equal wherever
the oracle's top-2 gap exceeds 4x that bound.  Reference semantics:
S/LlamaModel.swift:134-244, S/LlamaBlock.swift:178-276, S/GemmaBlock.swift:80-150.
"""
import os

import numpy as np
import pytest

from helpers import PageTables, forward_pair, gpu_model, oracle_twin
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu

LLAMA_8B_2L = dict(vocab_size=128256, d_model=4096, n_layers=2, n_heads=32, n_kv_heads=8, head_dim=128,
                   ffn_dim=14336, rope_theta=500000.0, rms_eps=1e-5, attn_cap=0.0, final_cap=0.0, window=0,
                   window_layer_parity=-1, act=abi.ACT_SILU, ref_compat=0)
GEMMA_9B_2L = dict(vocab_size=256000, d_model=3584, n_layers=2, n_heads=16, n_kv_heads=8, head_dim=256,
                   ffn_dim=14336, rope_theta=10000.0, rms_eps=1e-6, attn_cap=50.0, final_cap=30.0, window=4096,
                   window_layer_parity=0, act=abi.ACT_GELU_TANH, ref_compat=0)

CASES = {
    "llama8b": (LLAMA_8B_2L, 32, 5, (512, 2048)),
    "gemma9b": (GEMMA_9B_2L, 16, 4, (2048, 8192)),
}


def _copy_pool(pool, orc, cfg, blocks):
    """The device pool's pages (bf16, read back as fp32) into the oracle's pool."""
    L, Hkv, dh = cfg["n_layers"], cfg["n_kv_heads"], cfg["head_dim"]
    page = Hkv * 16 * dh
    for blk in blocks:
        for layer in range(L):
            for kv in (0, 1):
                base = ((blk * L + layer) * 2 + kv) * page
                orc.pool[base: base + page] = pool.read_page(blk, layer, kv).ravel()


@pytest.mark.parametrize("shape", sorted(CASES))
def test_full_width_verify_step(engine, oracle, shape):
    cfg, B, k, (lo, hi) = CASES[shape]
    rng = np.random.default_rng(2024)
    ctx = rng.integers(lo, hi + 1, B)
    n_new = k + 1
    nb = int(sum((c + n_new + 15) // 16 for c in ctx)) + 4
    m, pool = gpu_model(engine, cfg, abi.DTYPE_BF16, seed=5, num_blocks=nb, max_tokens=B * n_new + 64,
                        max_seqs=B)
    try:
        pool.fill_random(17, 1.0)
        orc = oracle_twin(oracle, m, cfg, nb, emulate_bf16=True, nthreads=os.cpu_count() or 8)
        pt = PageTables(nb)
        V = cfg["vocab_size"]
        batch = [(sid, rng.integers(0, V, n_new).tolist(), int(c)) for sid, c in enumerate(ctx)]
        for sid, _, c in batch:
            pt.reserve(sid, c + n_new)
        _copy_pool(pool, orc, cfg, sorted(b for t in pt.tables.values() for b in t))
        g, o = forward_pair(m, pool, orc, pt, batch, last_n=n_new)
        assert g.shape == (B * n_new, V)
        assert np.isfinite(g).all()
        scale = np.abs(o).max()
        err = np.abs(g - o).max() / scale
        assert err < 2e-2, f"{shape}: max |dlogit| / max|logit| = {err:.3e}"
        top2 = np.sort(o, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 4 * 2e-2 * scale
        assert (np.argmax(g, 1)[clear] == np.argmax(o, 1)[clear]).all()
        assert engine.device_error() == 0
    finally:
        pool.close()
        m.close()
