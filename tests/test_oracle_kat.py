"""Pins the CPU oracle to known answers (CPU only).

The reference has no tests or fixtures; tests/golden/sampler_kat.json holds the
published Philox4x32-10 vectors and hand-derived / independently restated
SpeculativeSampler answers (see tests/golden/make_golden.py).
"""
import json
from pathlib import Path

import numpy as np
import pytest

KAT = json.loads((Path(__file__).parent / "golden" / "sampler_kat.json").read_text())


def test_philox_published_vectors(oracle):
    for v in KAT["philox"]:
        assert oracle.philox(v["ctr"], v["key"]) == v["out"]


def test_uniform_coordinates(oracle):
    for v in KAT["uniform"]:
        u = oracle.uniform(*v["coord"])
        assert u == v["u"]
        assert 0.0 <= u < 1.0


def test_sample_from_probs(oracle):
    for c in KAT["sample_from_probs"]:
        assert oracle.sample_from_probs(c["probs"], c["r"]) == c["expect"], c["why"]


def test_verify_token(oracle):
    for c in KAT["verify_token"]:
        acc, tok = oracle.verify_token(c["d"], c["p"], c["q"], c["ra"], c["rr"])
        assert acc == c["accept"], c["why"]
        if not acc:
            assert tok == c["token"], c["why"]


def test_verify_sequence(oracle):
    for c in KAT["verify_sequence"]:
        out = oracle.verify_sequence_probs(c["drafts"], np.array(c["p"]), np.array(c["q"]), c["seed"], c["step"],
                                           c["seq"])
        assert out == c["expect"]


def test_softmax_matches_reference_formula(oracle):
    rng = np.random.default_rng(0)
    x = rng.normal(0, 2, 1000).astype(np.float32)
    p = oracle.softmax(x)
    e = np.exp((x - x.max()).astype(np.float64))
    np.testing.assert_allclose(p, e / e.sum(), rtol=2e-6, atol=1e-9)
    assert oracle.softmax(np.array([1.0, 1.0], np.float32)).tolist() == [0.5, 0.5]
    # temperature convention logits / T (S/Sampler.swift:19-23)
    np.testing.assert_array_equal(oracle.softmax(x, 0.8), oracle.softmax((x / np.float32(0.8)).astype(np.float32)))


def test_greedy_argmax_first_max_wins(oracle):
    # S/yanaiengine.swift sampler self-check: token 3 = 2.0 beats 7 = 1.8 ...
    logits = np.full(10, -10.0, np.float32)
    logits[[3, 7, 1, 5]] = [2.0, 1.8, 1.5, 1.0]
    tok, p = oracle.draft_sample(logits, 0.0, 1, 0, 0, 0)
    assert tok == 3 and p[3] == 1.0 and p.sum() == 1.0
    logits[8] = 2.0  # tie: first maximum wins (strict >, S/Sampler.swift:81-91)
    assert oracle.draft_sample(logits, 0.0, 1, 0, 0, 0)[0] == 3


@pytest.mark.parametrize("V,k", [(6, 3), (11, 4)])
def test_speculative_sampling_preserves_target_distribution(oracle, V, k):
    """Rejection sampling property: the first emitted token ~ target q, whatever p is."""
    rng = np.random.default_rng(V)
    q = rng.random((k + 1, V)).astype(np.float32) ** 2
    q /= q.sum(1, keepdims=True)
    p = rng.random((k, V)).astype(np.float32) ** 2
    p /= p.sum(1, keepdims=True)
    n = 30000
    counts = np.zeros(V)
    for step in range(n):
        d = [oracle.sample_from_probs(p[i], oracle.uniform(9, step, 0, i, 0)) for i in range(k)]
        out = oracle.verify_sequence_probs(d, p, q, 9, step, 0)
        counts[out[0]] += 1
    emp = counts / n
    assert np.abs(emp - q[0]).max() < 4 * np.sqrt(q[0].max() / n) + 1e-3
