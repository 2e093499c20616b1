"""Host-side arithmetic of bench.py (CPU only): the verify-forward roofline and the
launch-trace attribution it is timed from."""
from __future__ import annotations

import numpy as np
import pytest

import bench


def test_verify_roofline_bytes():
    cfg = bench.TARGET
    ctx = [512, 1000, 2048]
    k = 5
    peaks = {"hbm_gbs": 6000.0, "src": "test"}
    r = bench.verify_roofline(cfg, ctx, k, 1, 1000.0, peaks)
    kv_tok = 2 * cfg["n_kv_heads"] * cfg["head_dim"] * 2 * cfg["n_layers"]  # K and V, bf16, all layers
    assert r["kv_bytes"] == sum(c + k + 1 for c in ctx) * kv_tok
    assert r["weight_bytes"] == bench.params_bytes(cfg)  # one GPU: every weight, LM head included
    assert r["achieved_gbs"] == pytest.approx(r["bytes"] / 1e-3 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved_gbs"] / 6000.0)
    # a tensor-parallel shard streams its share of the layers' weights and KV heads plus the whole LM head
    r2 = bench.verify_roofline(cfg, ctx, k, 2, 1000.0, peaks)
    lm = cfg["vocab_size"] * cfg["d_model"] * 2
    assert r2["weight_bytes"] == pytest.approx((bench.params_bytes(cfg) - lm) / 2 + lm)
    assert r2["kv_bytes"] == r["kv_bytes"] / 2
    assert bench.verify_roofline(cfg, ctx, k, 1, None, peaks) is None


class _FakeEngine:
    """Replays launch-trace records (entry, start, end, kind) in ns."""

    def __init__(self, recs):
        self.recs = np.array(recs, dtype=np.uint64)
        self.n = 0

    def launches(self):
        return self.n

    def trace(self, cap):
        self.cap = cap

    def trace_read(self):
        out = np.zeros((self.cap, 4), np.uint64)
        out[: len(self.recs)] = self.recs
        self.n = len(self.recs)
        return out, self.n


class _FakeScheduler:
    def step(self):
        return 0


def test_trace_breakdown_verify_span():
    emb, ds, vf = 1, 5, 7
    gemm_qkv = 3 | (1 << 4) | (48 << 8) | (12 << 24)
    lm = 3 | (4 << 4) | (1002 << 8) | (12 << 24)
    recs = [  # draft forward tail, then the target forward, then verification
        (0, 100, 1_000, ds),
        (900, 3_000, 4_000, emb),      # target embedding: 2 us behind the sampler (hand-off)
        (3_500, 4_500, 10_000, gemm_qkv),
        (9_000, 10_500, 20_000, lm),   # LM head
        (19_000, 20_600, 30_000, vf),
    ]
    out = bench.trace_breakdown(_FakeEngine(recs), _FakeScheduler(), cap=16)
    # the last embedding's share (from the sampler's end) through the LM head's end
    assert out["verify_forward_us"] == pytest.approx((20_000 - 1_000) / 1e3)
    assert out["launches"] == 5
    assert out["count"]["embed"] == 1
    # idle = the part of each share before the first CTA got past the dependency wait
    assert out["idle_us"] == pytest.approx(((3_000 - 1_000) + (4_500 - 4_000) + 500 + 600) / 1e3)
