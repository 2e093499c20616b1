"""Verify forward (yk_forward_step) vs the fp32 oracle forward on the same weights.

Tolerances:
  fp32 model: max |dlogit| <= 2e-4 * max|logit| (accumulation order only);
  bf16 model vs the oracle emulating the bf16 storage points:
      max |dlogit| <= 2e-2 * max|logit| (accumulation order and P/rotation rounding);
  bf16 model vs the pure fp32 oracle: max |dlogit| <= 5e-2 * max|logit|.
Greedy tokens must agree wherever the oracle's top-2 gap exceeds the error bound.
"""
import numpy as np
import pytest

from helpers import TINY, PageTables, forward_pair, gpu_model, oracle_twin, step_inputs
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu
NB = 64


def _rel(g, o):
    return np.abs(g - o).max() / max(np.abs(o).max(), 1e-6)


def _greedy_agree(g, o, tol_abs):
    top2 = np.sort(o, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 4 * tol_abs
    assert (np.argmax(g, 1)[clear] == np.argmax(o, 1)[clear]).all()


def _drive(engine, oracle, cfg, dtype, emulate, tol, init_std=0.02, steps=3, k=4,
           prefill=((0, 17), (1, 40), (2, 5)), nb=NB, max_tokens=256):
    m, pool = gpu_model(engine, cfg, dtype, seed=3, num_blocks=nb, init_std=init_std, max_tokens=max_tokens)
    try:
        orc = oracle_twin(oracle, m, cfg, nb, emulate_bf16=emulate)
        pt = PageTables(nb)
        rng = np.random.default_rng(1)
        V = cfg["vocab_size"]
        lens = {0: 0, 1: 0, 2: 0}
        # ragged prefill: 3 sequences, by default 17 / 40 / 5 tokens (page-boundary crossings)
        batch = []
        for sid, n in prefill:
            batch.append((sid, rng.integers(0, V, n).tolist(), 0))
            lens[sid] = n
        g, o = forward_pair(m, pool, orc, pt, batch)
        assert np.isfinite(g).all()
        assert _rel(g, o) < tol, f"prefill rel err {_rel(g, o):.3e}"
        _greedy_agree(g, o, tol * np.abs(o).max())
        # verify-shaped steps: k+1 new tokens per sequence, logits for the last k+1
        for _ in range(steps):
            batch = []
            for sid in (0, 1, 2):
                batch.append((sid, rng.integers(0, V, k + 1).tolist(), lens[sid]))
                lens[sid] += k + 1
            g, o = forward_pair(m, pool, orc, pt, batch, last_n=k + 1)
            assert g.shape == (3 * (k + 1), V)
            assert _rel(g, o) < tol, f"step rel err {_rel(g, o):.3e}"
            _greedy_agree(g, o, tol * np.abs(o).max())
        # KV page contents (K stored rotated, V as projected)
        blk = pt.tables[1][0]
        for layer in range(cfg["n_layers"]):
            for kv in (0, 1):
                page = pool.read_page(blk, layer, kv)
                ref = _oracle_page(orc, cfg, blk, layer, kv)
                assert np.abs(page - ref).max() <= tol * max(np.abs(ref).max(), 1e-3) * 4
        assert engine.device_error() == 0
    finally:
        pool.close()
        m.close()


def _oracle_page(orc, cfg, blk, layer, kv):
    L, Hkv, dh = cfg["n_layers"], cfg["n_kv_heads"], cfg["head_dim"]
    per_layer = 2 * Hkv * 16 * dh
    base = blk * L * per_layer + layer * per_layer + kv * Hkv * 16 * dh
    return orc.pool[base: base + Hkv * 16 * dh].reshape(Hkv, 16, dh)


def test_fp32_tiny(engine, oracle):
    _drive(engine, oracle, TINY, abi.DTYPE_F32, False, 2e-4)


def test_bf16_tiny_vs_bf16_emulating_oracle(engine, oracle):
    _drive(engine, oracle, TINY, abi.DTYPE_BF16, True, 2e-2)


def test_bf16_long_ragged_prefill(engine, oracle):
    """Prefill inside the batch (the scheduler's first step feeds whole prompts,
    S/Scheduler.swift:68-69,201-202): 1150 tokens in one step -- several 256-token
    GEMM tiles, many 64-row attention query tiles per sequence, the RMSNorm kernels
    instead of the folded norm -- then verify steps on the long contexts."""
    _drive(engine, oracle, TINY, abi.DTYPE_BF16, True, 2e-2, steps=2,
           prefill=((0, 300), (1, 700), (2, 150)), nb=96, max_tokens=1216)


def test_wide_rows(engine, oracle):
    """d_model 8192, the 70B shape's rows: the RMSNorm kernel keeps the widest rows in
    registers (every norm unfused in fp32; the final norm's bf16 store in bf16)."""
    cfg = dict(TINY, d_model=8192, n_layers=1, n_heads=64, n_kv_heads=8, head_dim=128, ffn_dim=512)
    _drive(engine, oracle, cfg, abi.DTYPE_F32, False, 1e-3, steps=1)
    _drive(engine, oracle, cfg, abi.DTYPE_BF16, True, 2e-2, steps=1)


def test_bf16_tiny_vs_fp32_oracle(engine, oracle):
    _drive(engine, oracle, TINY, abi.DTYPE_BF16, False, 5e-2)


@pytest.mark.parametrize("dh", [128, 256])
def test_bf16_head_dims(engine, oracle, dh):
    cfg = dict(TINY, head_dim=dh, n_heads=4, n_kv_heads=1)
    _drive(engine, oracle, cfg, abi.DTYPE_BF16, True, 2e-2, steps=2)


def test_gemma_variant(engine, oracle):
    """GeGLU, attention cap 50, final cap 30, window 8 on even layers, head_dim 256, eps 1e-6."""
    cfg = dict(TINY, act=abi.ACT_GELU_TANH, attn_cap=50.0, final_cap=30.0, window=8, window_layer_parity=0,
               head_dim=256, n_heads=2, n_kv_heads=1, rms_eps=1e-6)
    _drive(engine, oracle, cfg, abi.DTYPE_BF16, True, 2e-2, init_std=0.08, steps=3)


def test_gemma_variant_fp32(engine, oracle):
    cfg = dict(TINY, act=abi.ACT_GELU_TANH, attn_cap=5.0, final_cap=3.0, window=8, window_layer_parity=0,
               head_dim=128, n_heads=4, n_kv_heads=2, rms_eps=1e-6)
    _drive(engine, oracle, cfg, abi.DTYPE_F32, False, 2e-4, init_std=0.08, steps=3)


def test_ref_compat(engine, oracle):
    """bias 0.1 + ReLU on every projection and LM-head cap 30 (S/LinearLayer.swift:61,99-121)."""
    cfg = dict(TINY, ref_compat=1)
    _drive(engine, oracle, cfg, abi.DTYPE_F32, False, 2e-4, steps=2)


def test_rejects_bad_block_id(engine):
    m, pool = gpu_model(engine, TINY, abi.DTYPE_BF16, seed=1, num_blocks=4)
    try:
        with pytest.raises(abi.YKError) as ei:
            m.forward(pool, [1, 2, 3], [0, 3], [3], np.array([[7]], np.int32))
        assert ei.value.status == abi.YK_ERR_ARG
        with pytest.raises(abi.YKError):
            m.forward(pool, [1, 2, 10**6], [0, 3], [3], np.array([[0]], np.int32))
    finally:
        pool.close()
        m.close()


@pytest.mark.parametrize("knobs", [
    {"YK_GEMM_PUSH_MIN": "0"},   # cluster split-K, copy-engine exchange (QKV RoPE rows staged)
    {"YK_GEMM_VARIANT": "8"},    # cluster split-K, distributed-shared-memory loads
    {"YK_GEMM_VARIANT": "32"},   # no clusters: whole tiles straight from the accumulator
    {"YK_GEMM_VARIANT": "33"},   # no clusters, pure stream-K: cut tiles finished by the last arriver
    {"YK_FUSE_NORM": "0"},       # RMSNorm as separate kernels
    {"YK_GEMM_CHAIN": "1"},      # gate/up and down_proj as one launch with a grid barrier
    {"YK_GEMM_CHAIN": "1", "YK_FUSE_NORM": "0"},
])
def test_bf16_gemm_paths_with_fused_norm(oracle, monkeypatch, knobs):
    """The bf16 forward through every GEMM work split and reduction, each carrying
    the RMSNorm folded into the residual epilogue (x = bf16(h * gain), 32-row sums
    of squares) and the next GEMM (1/rms per token), and with the norm unfused."""
    for k, v in knobs.items():
        monkeypatch.setenv(k, v)
    e = abi.Engine(0)  # reads the knobs at creation
    try:
        # 6 query heads x 128: o_proj has K = 768 (12 k-blocks over 2 tiles), so pure
        # stream-K cuts its tiles and the residual epilogue runs in the last arriver
        cfg = dict(TINY, head_dim=128, n_heads=6, n_kv_heads=2)
        _drive(e, oracle, cfg, abi.DTYPE_BF16, True, 2e-2, steps=2)
    finally:
        e.close()


def test_gemma_split_pools_vs_single_pool_oracle(engine, oracle):
    """Split pools (yk_forward_step_split): the global layers' K/V in one pool, the
    windowed layers' in another, each with its own page tables (different block
    assignments), against the oracle's single pool: same logits within the bf16
    bound, prefill and verify steps."""
    cfg = dict(TINY, act=abi.ACT_GELU_TANH, attn_cap=50.0, final_cap=30.0, window=8, window_layer_parity=0,
               head_dim=256, n_heads=2, n_kv_heads=1, rms_eps=1e-6)
    c = abi.make_config(**cfg, dtype=abi.DTYPE_BF16, max_tokens=256, max_seqs=16)
    m = abi.Model(engine, c, seed=3, init_std=0.08)
    pg = abi.KVPool(engine, c, NB, abi.POOL_GLOBAL_LAYERS)
    pw = abi.KVPool(engine, c, NB, abi.POOL_WINDOWED_LAYERS)
    try:
        orc = oracle_twin(oracle, m, cfg, NB, emulate_bf16=True)
        pto, ptg, ptw = PageTables(NB), PageTables(NB), PageTables(NB)
        ptw.free = list(np.random.default_rng(5).permutation(NB))  # a different block assignment
        rng = np.random.default_rng(2)
        V = cfg["vocab_size"]
        lens = {0: 17, 1: 40, 2: 5}
        steps = [[(sid, rng.integers(0, V, n).tolist(), 0) for sid, n in lens.items()]]
        for _ in range(3):
            st = []
            for sid in (0, 1, 2):
                st.append((sid, rng.integers(0, V, 5).tolist(), lens[sid]))
                lens[sid] += 5
            steps.append(st)
        for i, batch in enumerate(steps):
            last_n = 0 if i == 0 else 5
            toks, qs, ctx, bt_o = step_inputs(pto, batch)
            bt_g = step_inputs(ptg, batch)[3]
            bt_w = step_inputs(ptw, batch)[3]
            rows = m.forward_split(pg, pw, toks, qs, ctx, bt_g, bt_w, last_n)
            g = m.logits(0, rows)
            o = orc.forward(toks, qs, ctx, bt_o, last_n)
            assert np.isfinite(g).all()
            assert _rel(g, o) < 2e-2, f"step {i}: rel err {_rel(g, o):.3e}"
        # the pools hold only their own layers
        with pytest.raises(abi.YKError):
            pw.read_page(0, 1, 0)  # layer 1 is global
        with pytest.raises(abi.YKError):
            m.forward(pg, toks, qs, ctx, bt_g, 5)  # a one-kind pool needs the split entry
        assert engine.device_error() == 0
    finally:
        pw.close()
        pg.close()
        m.close()
