"""Fused rejection sampler vs the oracle.

Bit-exact contract: identical probability tensors + identical (Philox) uniforms
give identical acceptance decisions and emitted tokens (yk_spec_verify_probs).
Logits entry points: the probabilities are computed on the device (expf and a
parallel max/sum), so they are compared with the reference softmax within a
tolerance; given the device's own p and q rows (read back), every decision and
token is compared bit-exactly.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu
KAT = json.loads((Path(__file__).parent / "golden" / "sampler_kat.json").read_text())


def test_golden_verify_sequences(engine):
    for c in KAT["verify_sequence"]:
        s = abi.Sampler(engine, 1, c["k"], c["V"])
        try:
            out, cnt = s.verify_probs(np.array(c["p"])[None], np.array(c["q"])[None], [c["drafts"]], c["seed"],
                                      c["step"], [c["seq"]])
        finally:
            s.close()
        assert out[0, : cnt[0]].tolist() == c["expect"]


def _sampler_probs(oracle, B, k, V, seed):
    rng = np.random.default_rng(seed)
    dl = rng.normal(0, 2.0, (B, k, V)).astype(np.float32)
    tl = rng.normal(0, 2.0, (B, k + 1, V)).astype(np.float32)
    p = np.stack([np.stack([oracle.softmax(dl[b, j]) for j in range(k)]) for b in range(B)])
    q = np.stack([np.stack([oracle.softmax(tl[b, j]) for j in range(k + 1)]) for b in range(B)])
    drafts = np.array([[oracle.sample_from_probs(p[b, j], oracle.uniform(seed, 3, b, j, 0)) for j in range(k)]
                       for b in range(B)], np.uint32)
    return p, q, drafts


def test_verify_probs_bit_exact_64x4x128256(engine, oracle):
    """Sampler shapes of the 8B/1B workload at 64 sequences: k=4, V=128256, N(0, 2^2) logits."""
    B, k, V = 64, 4, 128256
    p, q, drafts = _sampler_probs(oracle, B, k, V, 1234)
    seq_ids = np.arange(B, dtype=np.uint32)
    s = abi.Sampler(engine, B, k, V)
    try:
        for step in (3, 4):
            out, cnt = s.verify_probs(p, q, drafts, 1234, step, seq_ids)
            ref_out, ref_cnt = oracle.verify_batch_probs(drafts, p, q, 1234, step, seq_ids)
            np.testing.assert_array_equal(cnt, ref_cnt)
            for b in range(B):
                assert out[b, : cnt[b]].tolist() == ref_out[b, : ref_cnt[b]].tolist(), f"seq {b}"
    finally:
        s.close()


def test_verify_probs_edge_cases(engine, oracle):
    """Rows built to hit every branch of verifyToken / sampleFromProbs."""
    k, V = 4, 4099
    rng = np.random.default_rng(7)
    rows_p, rows_q, drafts = [], [], []
    for case in range(12):
        p = rng.random((k, V)).astype(np.float32) ** 4
        q = rng.random((k + 1, V)).astype(np.float32) ** 4
        p /= p.sum(1, keepdims=True)
        q /= q.sum(1, keepdims=True)
        d = rng.integers(0, V, k)
        if case == 0:
            q[:k] = p                      # ratio 1: all accepted, bonus
        if case == 1:
            p[:, d] = 0.0                  # p[d] = 0 -> ratio inf -> accept
        if case == 2:
            p[0, d[0]] = 0.0
            q[0, d[0]] = 0.0               # 0/0 -> NaN -> reject
        if case == 3:
            q[0] = p[0] * 0.5              # residual sums to 0 -> fallback to q
        if case == 4:
            q[0] = 0.0
            q[0, -1] = 1e-30               # residual concentrated on the last index
            p[0, d[0]] = 1.0
        if case == 5:
            q[k] *= 0.5                    # bonus cdf short of r -> fallback V-1 often
            q[:k] = p
        if case == 6:
            q[1] = np.float32(1.0 / V)     # exact ties everywhere
            p[1] = np.float32(1.0 / V)
            p[1, d[1]] = np.float32(2.0 / V)
        rows_p.append(p)
        rows_q.append(q)
        drafts.append(d)
    p = np.stack(rows_p).astype(np.float32)
    q = np.stack(rows_q).astype(np.float32)
    drafts = np.stack(drafts).astype(np.uint32)
    B = p.shape[0]
    seq_ids = np.arange(100, 100 + B, dtype=np.uint32)
    s = abi.Sampler(engine, B, k, V)
    try:
        for step in range(6):
            out, cnt = s.verify_probs(p, q, drafts, 99, step, seq_ids)
            ref_out, ref_cnt = oracle.verify_batch_probs(drafts, p, q, 99, step, seq_ids)
            np.testing.assert_array_equal(cnt, ref_cnt)
            np.testing.assert_array_equal(np.where(np.arange(k + 1)[None] < cnt[:, None], out, 0),
                                          np.where(np.arange(k + 1)[None] < ref_cnt[:, None], ref_out, 0))
    finally:
        s.close()


@pytest.mark.parametrize("B,T", [(16, 1.0), (16, 0.8), (16, 0.0), (64, 1.0)])
def test_sample_logits_matches_oracle(engine, oracle, B, T):
    """Whole sampler phase from logits; (64, 1.0) is the sampler-only workload's shape
    (64 sequences, k=4, V=128256, N(0, 2^2) logits, T=1)."""
    k, V = 4, 128256
    rng = np.random.default_rng(11)
    dl = rng.normal(0, 2.0, (B, k, V)).astype(np.float32)
    tl = rng.normal(0, 2.0, (B, k + 1, V)).astype(np.float32)
    seq_ids = np.arange(B, dtype=np.uint32)
    s = abi.Sampler(engine, B, k, V)
    try:
        drafts, out, cnt = s.sample_logits(dl, tl, T, 5, 1, seq_ids)
        p_dev = np.stack([np.stack([s.read_probs(b, j) for j in range(k)]) for b in range(B)])
        s_q = s.target_probs(B, T) if T > 0 else None
    finally:
        s.close()
    if T <= 0:  # greedy is exact end to end
        r_drafts, r_out, r_cnt = oracle.spec_sample_batch(dl, tl, T, 5, 1, seq_ids)
        np.testing.assert_array_equal(drafts, r_drafts)
        np.testing.assert_array_equal(cnt, r_cnt)
        for b in range(B):
            assert out[b, : cnt[b]].tolist() == r_out[b, : r_cnt[b]].tolist()
        assert (p_dev.max(-1) == 1.0).all() and (p_dev.sum(-1) == 1.0).all()
        return
    # Device probabilities vs the reference softmax.  The reference normalises by a
    # sequential fp32 sum of 128256 terms (relative error ~1e-5); the device sums in a
    # tree, so the two agree to 3e-4 relative, and CDF positions may shift by a few ids.
    for b in range(B):
        for j in range(k):
            np.testing.assert_allclose(p_dev[b, j], oracle.softmax(dl[b, j], T), rtol=3e-4, atol=1e-12)
    # Given the device's own probabilities, draft sampling is bit-exact.
    for b in range(B):
        for j in range(k):
            assert drafts[b, j] == oracle.sample_from_probs(p_dev[b, j], oracle.uniform(5, 1, b, j, 0))
    # Verification on the device's own p and q (q read back exactly as verification
    # formed it from the logits): decisions and tokens bit-exact against the oracle.
    q_dev = s_q
    r_out, r_cnt = oracle.verify_batch_probs(drafts, p_dev, q_dev, 5, 1, seq_ids)
    np.testing.assert_array_equal(cnt, r_cnt)
    for b in range(B):
        assert out[b, : cnt[b]].tolist() == r_out[b, : r_cnt[b]].tolist(), f"seq {b}"
    # and q itself is the reference softmax within the normalisation tolerance
    for b in range(B):
        for i in range(k + 1):
            np.testing.assert_allclose(q_dev[b, i], oracle.softmax(tl[b, i], T), rtol=3e-4, atol=1e-12)


def _stress_rows(rng, V):
    """Probability rows that drive the exact chain through its special cases."""
    rows = []
    r = rng.integers(0, 16, V).astype(np.float32) / np.float32(4096)  # dyadic: frequent rounding ties
    rows.append(r)
    r = rng.random(V).astype(np.float32)
    r[:3000] = 0.0                                                    # long +0 prefix
    rows.append(r)
    r = rng.random(V).astype(np.float32)
    r[:200] = np.float32(1e-30)                                       # tiny head (c below 2^-100)
    rows.append(r)
    r = (10.0 ** rng.uniform(-20, 0, V)).astype(np.float32)           # huge dynamic range
    rows.append(r)
    r = np.full(V, 1e-8, np.float32)
    r[V // 3] = 0.9                                                   # one dominant value mid-row
    rows.append(r)
    r = rng.random(V).astype(np.float32)
    r[::7] = np.float32(1e-40)                                        # subnormals sprinkled in
    rows.append(r)
    r = np.zeros(V, np.float32)
    r[-1] = 1.0                                                       # all mass on the last id
    rows.append(r)
    r = rng.random(V).astype(np.float32) * np.float32(0.5) / np.float32(V)  # sums to ~0.25: CDF fallback
    rows.append(r)
    return [x / np.float32(x.sum(dtype=np.float64)) if i not in (7,) else x for i, x in enumerate(rows)]


def test_chain_exact_on_adversarial_rows(engine, oracle):
    """Residual normaliser, residual CDF and bonus CDF on rows built to hit binade
    crossings, ties, zero/tiny/subnormal states: bit-exact against the oracle."""
    V, k = 20011, 1
    rng = np.random.default_rng(77)
    rows = _stress_rows(rng, V)
    P, Q, D = [], [], []
    for i, q0 in enumerate(rows):
        for mode in range(3):
            p = rng.random((k, V)).astype(np.float32)
            p /= p.sum(dtype=np.float64)
            q = np.stack([q0, rows[(i + 3) % len(rows)]]).astype(np.float32)
            d = int(rng.integers(V))
            if mode == 0:      # reject at position 0: residual chain over max(0, q - p)
                p[0, d] = 1.0
                q[0, d] = 0.0
            elif mode == 1:    # accept everything: bonus chain over q[1]
                p[0] = q[0]
            else:              # residual sums to zero: fallback to q
                p[0] = np.maximum(q[0], p[0])
                p[0, d] = 1.0
                q[0, d] = 0.0
            P.append(p)
            Q.append(q)
            D.append([d])
    P, Q, D = np.stack(P), np.stack(Q), np.array(D, np.uint32)
    B = P.shape[0]
    seq = np.arange(B, dtype=np.uint32)
    s = abi.Sampler(engine, B, k, V)
    try:
        for step in range(4):
            out, cnt = s.verify_probs(P, Q, D, 2024, step, seq)
            r_out, r_cnt = oracle.verify_batch_probs(D, P, Q, 2024, step, seq)
            np.testing.assert_array_equal(cnt, r_cnt)
            for b in range(B):
                assert out[b, : cnt[b]].tolist() == r_out[b, : r_cnt[b]].tolist(), f"row {b} step {step}"
    finally:
        s.close()
