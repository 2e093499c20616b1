"""Paged attention over long synthetic contexts, through yk_forward_step.

The KV pool is filled with N(0, 1) values on the device and copied into the
oracle's pool, so one verify step attends over hundreds of cached keys per
sequence.  The cases cover: items longer than the page ring (every head dim),
many key splits merged by the last CTA of a group, one and two query m-tiles,
windowed + soft-capped layers.  Tolerance as for the bf16 forward:
max |dlogit| <= 2e-2 * max |logit| against the bf16-emulating oracle.
"""
import numpy as np
import pytest

from helpers import TINY, PageTables, forward_pair, gpu_model, oracle_twin
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu

CASES = [
    # dh, G, n_kv_heads, sequences, new tokens, extra config
    (64, 4, 16, 32, 1, {}),                      # many spans: whole contexts per item, ring of 12 wraps
    (128, 4, 16, 32, 6, {}),                     # verify shape (24 rows = 2 m-tiles), ring of 8 wraps
    (128, 4, 2, 4, 6, {}),                       # few spans: many splits merged by the last CTA
    (64, 1, 2, 3, 1, {}),                        # one query row per item
    (256, 2, 4, 8, 3, {}),                       # head dim 256, ring of 4 wraps
    (128, 2, 8, 16, 4, dict(window=100, window_layer_parity=0, attn_cap=30.0)),
]


@pytest.mark.parametrize("dh,G,hkv,nseq,new,extra", CASES)
def test_bf16_long_context(engine, oracle, dh, G, hkv, nseq, new, extra):
    cfg = dict(TINY, head_dim=dh, n_kv_heads=hkv, n_heads=hkv * G, **extra)
    rng = np.random.default_rng(dh * 1000 + hkv * 10 + nseq)
    ctx = rng.integers(150, 700, nseq)
    nb = int(sum((c + new + 15) // 16 for c in ctx)) + 4
    m, pool = gpu_model(engine, cfg, abi.DTYPE_BF16, seed=5, num_blocks=nb, max_tokens=max(64, nseq * new),
                        max_seqs=nseq)
    try:
        pool.fill_random(11, 1.0)
        orc = oracle_twin(oracle, m, cfg, nb, emulate_bf16=True)
        pt = PageTables(nb)
        L = cfg["n_layers"]
        per_layer = 2 * hkv * 16 * dh
        for sid in range(nseq):
            pt.reserve(sid, int(ctx[sid]))
            for blk in pt.tables[sid]:
                for layer in range(L):
                    for kv in (0, 1):
                        base = blk * L * per_layer + layer * per_layer + kv * hkv * 16 * dh
                        orc.pool[base: base + hkv * 16 * dh] = pool.read_page(blk, layer, kv).ravel()
        V = cfg["vocab_size"]
        batch = [(sid, rng.integers(0, V, new).tolist(), int(ctx[sid])) for sid in range(nseq)]
        g, o = forward_pair(m, pool, orc, pt, batch, last_n=new)
        assert np.isfinite(g).all()
        err = np.abs(g - o).max() / np.abs(o).max()
        assert err < 2e-2, f"rel err {err:.3e}"
        assert engine.device_error() == 0
    finally:
        pool.close()
        m.close()
