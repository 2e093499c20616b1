"""Shared helpers for the GPU parity tests: a GPU model plus an oracle twin that
holds exactly the same weights (read back from the device)."""
from __future__ import annotations

import numpy as np

from yanaiengine_b200 import abi

TINY = dict(vocab_size=512, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=384,
            rope_theta=10000.0, rms_eps=1e-5, attn_cap=0.0, final_cap=0.0, window=0, window_layer_parity=-1,
            act=abi.ACT_SILU, ref_compat=0)

# Small fp32 speculative workload: a d=2048, 8-layer target and a d=512, 4-layer draft (V=32000).
SMALL_F32_TARGET = dict(vocab_size=32000, d_model=2048, n_layers=8, n_heads=32, n_kv_heads=8, head_dim=64, ffn_dim=5632,
                 rope_theta=10000.0, rms_eps=1e-5, attn_cap=0.0, final_cap=0.0, window=0, window_layer_parity=-1,
                 act=abi.ACT_SILU, ref_compat=0)
SMALL_F32_DRAFT = dict(SMALL_F32_TARGET, d_model=512, n_layers=4, n_heads=8, n_kv_heads=2, ffn_dim=1408)


def gpu_model(engine, cfg: dict, dtype: int, seed: int, num_blocks: int, max_tokens: int = 256, max_seqs: int = 16,
              init_std: float = 0.02):
    c = abi.make_config(**cfg, dtype=dtype, max_tokens=max_tokens, max_seqs=max_seqs)
    m = abi.Model(engine, c, seed=seed, init_std=init_std)
    pool = abi.KVPool(engine, c, num_blocks)
    return m, pool


def oracle_twin(oracle_mod, model: abi.Model, cfg: dict, num_blocks: int, emulate_bf16: bool, nthreads: int = 8):
    L = cfg["n_layers"]
    w = dict(embed=model.get(abi.T_EMBED), lm_head=model.get(abi.T_LM_HEAD), final_norm=model.get(abi.T_FINAL_NORM))
    for name, t in (("wq", abi.T_WQ), ("wk", abi.T_WK), ("wv", abi.T_WV), ("wo", abi.T_WO), ("wg", abi.T_WGATE),
                    ("wu", abi.T_WUP), ("wd", abi.T_WDOWN), ("n1", abi.T_NORM1), ("n2", abi.T_NORM2)):
        w[name] = [model.get(t, l) for l in range(L)]
    return oracle_mod.OracleModel(cfg, w, num_blocks, emulate_bf16=emulate_bf16, nthreads=nthreads)


class PageTables:
    """Minimal page-table bookkeeping for driving both forwards identically."""

    def __init__(self, num_blocks: int):
        self.free = list(range(num_blocks - 1, -1, -1))
        self.tables: dict[int, list[int]] = {}

    def reserve(self, seq: int, n: int):
        t = self.tables.setdefault(seq, [])
        while len(t) * 16 < n:
            t.append(self.free.pop())

    def matrix(self, seqs):
        mb = max(1, max(len(self.tables.get(s, [])) for s in seqs))
        out = np.zeros((len(seqs), mb), np.int32)
        for i, s in enumerate(seqs):
            t = self.tables.get(s, [])
            out[i, : len(t)] = t
        return out


def step_inputs(pt: PageTables, batch: list[tuple[int, list[int], int]]):
    """batch: (seq_id, new tokens, cache length before) -> forward-step arrays."""
    toks, qs, ctx, seqs = [], [0], [], []
    for sid, new, before in batch:
        pt.reserve(sid, before + len(new))
        toks += list(new)
        qs.append(len(toks))
        ctx.append(before + len(new))
        seqs.append(sid)
    return toks, qs, ctx, pt.matrix(seqs)


def forward_pair(gpu_model_, gpu_pool, orc, pt: PageTables, batch, last_n: int = 0):
    """Runs the same ragged step through the CUDA module and the oracle."""
    toks, qs, ctx, bt = step_inputs(pt, batch)
    rows = gpu_model_.forward(gpu_pool, toks, qs, ctx, bt, last_n)
    g = gpu_model_.logits(0, rows)
    o = orc.forward(toks, qs, ctx, bt, last_n)
    return g, o
