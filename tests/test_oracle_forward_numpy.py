"""Pins the oracle's paged forward to an independent numpy restatement (CPU only).

The numpy model below recomputes every step from the whole token history (no
KV cache, no pages): causal attention over positions 0..p, RoPE on interleaved
pairs with denominators theta^(2i/dh) (S/gemm.metal:674-682), RMSNorm
x * rsqrt(mean(x^2) + eps) * g (S/gemm.metal:377-401), the windowed layers and
score cap of batched_paged_attention_kernel (S/gemm.metal:572, 604-606), the
SiLU / tanh-GELU gated MLP (S/gemm.metal:231-241, 405-413;
S/LlamaBlock.swift:264-267), and the final norm, LM head and final cap
(S/LlamaModel.swift:225, S/LMHead.swift:20-34). The oracle instead writes K/V
into a paged pool across ragged multi-sequence steps and reads them back
through block tables, so agreement pins its cache layout and position formula
as well as its arithmetic. Tolerance: fp32 vs float64, |diff| <= 2e-4 * max|logit| + 2e-5.
"""
from __future__ import annotations

import numpy as np
import pytest

BASE = dict(vocab_size=97, d_model=48, n_layers=3, n_heads=4, n_kv_heads=2, head_dim=12, ffn_dim=80,
            rope_theta=10000.0, rms_eps=1e-5, attn_cap=0.0, final_cap=0.0, window=0, window_layer_parity=-1,
            act=0, ref_compat=0)

CASES = {
    "llama_silu_gqa": BASE,
    "gemma_gelu_window_caps": dict(BASE, act=1, attn_cap=1.5, final_cap=3.0, window=5, window_layer_parity=0),
    "window_all_layers_mha": dict(BASE, n_kv_heads=4, window=7, window_layer_parity=-1, rope_theta=500.0),
    "ref_compat_relu_bias": dict(BASE, ref_compat=1),
}


def weights(cfg, seed):
    r = np.random.default_rng(seed)
    d, H, Hk, dh, F, V, L = (cfg[k] for k in ("d_model", "n_heads", "n_kv_heads", "head_dim", "ffn_dim",
                                               "vocab_size", "n_layers"))
    g = lambda *s: (r.standard_normal(s) * 0.3).astype(np.float32)  # noqa: E731
    w = dict(embed=g(V, d), lm_head=g(V, d), final_norm=(1 + 0.2 * r.standard_normal(d)).astype(np.float32))
    w["wq"] = [g(H * dh, d) for _ in range(L)]
    w["wk"] = [g(Hk * dh, d) for _ in range(L)]
    w["wv"] = [g(Hk * dh, d) for _ in range(L)]
    w["wo"] = [g(d, H * dh) for _ in range(L)]
    w["wg"] = [g(F, d) for _ in range(L)]
    w["wu"] = [g(F, d) for _ in range(L)]
    w["wd"] = [g(d, F) for _ in range(L)]
    w["n1"] = [(1 + 0.2 * r.standard_normal(d)).astype(np.float32) for _ in range(L)]
    w["n2"] = [(1 + 0.2 * r.standard_normal(d)).astype(np.float32) for _ in range(L)]
    return w


def numpy_forward(cfg, w, tokens):
    """All-position logits of one sequence, float64, recomputed from scratch."""
    d, H, Hk, dh = cfg["d_model"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    compat = cfg["ref_compat"] != 0
    n = len(tokens)
    W64 = {k: ([np.float64(x) for x in v] if isinstance(v, list) else np.float64(v)) for k, v in w.items()}

    def rms(x, g):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + cfg["rms_eps"]) * g

    def lin(x, m, relu=False):
        y = x @ m.T
        if compat and relu:
            y = np.maximum(y + 0.1, 0.0)
        return y

    pos = np.arange(n, dtype=np.float64)
    inv = cfg["rope_theta"] ** (-(2.0 * np.arange(dh // 2)) / dh)
    ang = pos[:, None] * inv[None, :]
    cs, sn = np.cos(ang), np.sin(ang)

    def rope(x):  # x: [n, heads, dh], interleaved pairs (2i, 2i+1)
        x0, x1 = x[..., 0::2], x[..., 1::2]
        out = np.empty_like(x)
        out[..., 0::2] = x0 * cs[:, None, :] - x1 * sn[:, None, :]
        out[..., 1::2] = x0 * sn[:, None, :] + x1 * cs[:, None, :]
        return out

    h = W64["embed"][np.asarray(tokens)]
    i, j = np.arange(n)[:, None], np.arange(n)[None, :]
    for l in range(cfg["n_layers"]):
        xn = rms(h, W64["n1"][l])
        q = rope(lin(xn, W64["wq"][l], True).reshape(n, H, dh))
        k = rope(lin(xn, W64["wk"][l], True).reshape(n, Hk, dh))
        v = lin(xn, W64["wv"][l], True).reshape(n, Hk, dh)
        windowed = cfg["window"] > 0 and (cfg["window_layer_parity"] < 0 or l % 2 == cfg["window_layer_parity"])
        mask = j <= i
        if windowed:
            mask &= (i - j) < cfg["window"]
        att = np.empty((n, H, dh))
        for hq in range(H):
            kv = hq // (H // Hk)
            s = (q[:, hq, :] @ k[:, kv, :].T) / np.sqrt(dh)
            if cfg["attn_cap"] > 0:
                s = cfg["attn_cap"] * np.tanh(s / cfg["attn_cap"])
            s = np.where(mask, s, -np.inf)
            p = np.exp(s - s.max(-1, keepdims=True))
            att[:, hq, :] = (p / p.sum(-1, keepdims=True)) @ v[:, kv, :]
        h = h + lin(att.reshape(n, H * dh), W64["wo"][l], True)
        xn = rms(h, W64["n2"][l])
        gt, up = lin(xn, W64["wg"][l], True), lin(xn, W64["wu"][l], True)
        if cfg["act"] == 1:
            a = 0.5 * gt * (1 + np.tanh(np.sqrt(2 / np.pi) * (gt + 0.044715 * gt ** 3)))
        else:
            a = gt / (1 + np.exp(-gt))
        h = h + lin(a * up, W64["wd"][l], True)
    z = rms(h, W64["final_norm"]) @ W64["lm_head"].T
    fcap = 30.0 if compat else cfg["final_cap"]
    if compat:
        z = z + 0.1
    if fcap > 0:
        z = fcap * np.tanh(z / fcap)
    return z


def _close(got, want, what):
    tol = 2e-4 * float(np.abs(want).max()) + 2e-5
    err = float(np.abs(got - want).max())
    assert err <= tol, f"{what}: max |diff| {err:.3g} > {tol:.3g}"


class Pages:
    def __init__(self, nb, bs=16):
        self.free, self.bs, self.tab = list(range(nb - 1, -1, -1)), bs, {}

    def table(self, seqs, lens):
        for s, n in zip(seqs, lens):
            t = self.tab.setdefault(s, [])
            while len(t) * self.bs < n:
                # Hand pages out in a scattered order so contiguity is never assumed.
                t.append(self.free.pop(len(self.free) // 2))
        mb = max(len(self.tab[s]) for s in seqs)
        out = np.zeros((len(seqs), mb), np.int32)
        for r, s in enumerate(seqs):
            out[r, : len(self.tab[s])] = self.tab[s]
        return out


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_forward_matches_numpy(oracle, name):
    cfg = CASES[name]
    w = weights(cfg, seed=sorted(CASES).index(name) + 11)
    rng = np.random.default_rng(5)
    nb = 24
    orc = oracle.OracleModel(cfg, w, nb, emulate_bf16=False, nthreads=4)
    pages = Pages(nb)
    # Three sequences, ragged steps: prefills of different lengths, then draft-
    # verify-sized chunks and single-token decodes, interleaved in one batch.
    hist = {s: [] for s in range(3)}
    steps = [{0: 19, 1: 5, 2: 33}, {0: 4, 1: 1, 2: 5}, {1: 20}, {0: 1, 2: 3, 1: 4}, {0: 17, 2: 1}]
    for st, chunk in enumerate(steps):
        seqs = sorted(chunk)
        toks, qs = [], [0]
        for s in seqs:
            new = rng.integers(0, cfg["vocab_size"], chunk[s]).tolist()
            hist[s] += new
            toks += new
            qs.append(len(toks))
        lens = [len(hist[s]) for s in seqs]
        bt = pages.table(seqs, lens)
        got = orc.forward(toks, qs, lens, bt, last_n=0)
        r0 = 0
        for s in seqs:
            n_new = chunk[s]
            want = numpy_forward(cfg, w, hist[s])[-n_new:]
            _close(got[r0:r0 + n_new], want, f"{name} step {st} seq {s}")
            r0 += n_new
        # last_n selects the trailing rows of each sequence.
        if st == 1:
            tail = orc.forward(toks, qs, lens, bt, last_n=2)
            ref = np.concatenate([got[qs[i]:qs[i + 1]][-2:] for i in range(len(seqs))])
            np.testing.assert_array_equal(tail, ref)


def test_numpy_restatement_sees_window_and_caps(oracle):
    """Guards against a vacuous pin: window, caps and GELU each change the logits."""
    toks = list(np.random.default_rng(1).integers(0, 97, 30))
    w = weights(BASE, 3)
    base = numpy_forward(BASE, w, toks)
    for k, v in (("window", 4), ("attn_cap", 0.5), ("final_cap", 1.0), ("act", 1)):
        assert np.abs(numpy_forward(dict(BASE, **{k: v}), w, toks) - base).max() > 1e-3, k
