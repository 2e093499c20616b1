"""Generates tests/golden/sampler_kat.json -- known answers for the sampler path.

The reference ships no tests, fixtures or golden vectors and cannot run here
(Swift + Metal), so the known answers come from two independent sources:
  * Philox4x32-10 known-answer vectors published with Salmon et al. (SC'11,
    Random123 kat_vectors), copied as numbers;
  * cases derived by hand from the reference source
    (Sources/yanaiengine/SpeculativeSampler.swift), each with the reasoning in
    its "why" field, plus random cases evaluated by the pure-Python restatement
    below (numpy float32 scalar arithmetic: one rounding per + - * /, which is
    exact IEEE fp32 because float64 intermediates round innocuously).
This script does not import the oracle or the CUDA module.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

F = np.float32
OUT = Path(__file__).resolve().parent / "sampler_kat.json"

PHILOX_KAT = [
    # (counter[4], key[2]) -> out[4]; Philox4x32-10 vectors of the Random123 distribution
    ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
    ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
    ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
     [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
]


def philox(ctr, key):
    c = list(ctr)
    k = list(key)
    M = 0xFFFFFFFF
    for _ in range(10):
        p0 = 0xD2511F53 * c[0]
        p1 = 0xCD9E8D57 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k[0]) & M, p1 & M, ((p0 >> 32) ^ c[3] ^ k[1]) & M, p0 & M]
        k = [(k[0] + 0x9E3779B9) & M, (k[1] + 0xBB67AE85) & M]
    return c


def uniform(seed, step, seq, pos, slot) -> float:
    w = philox([step, seq, pos, slot], [seed & 0xFFFFFFFF, seed >> 32])[0]
    return float(F(w >> 8) * F(1.0 / 16777216.0))


# --- pure-Python restatement of SpeculativeSampler.swift (fp32) --------------
def sample_from_probs(probs, r):           # :63-73
    cdf = F(0)
    r = F(r)
    for i, p in enumerate(probs):
        cdf = F(cdf + F(p))
        if r <= cdf:
            return i
    return len(probs) - 1


def verify_token(d, p, q, ra, rr):          # :20-60
    ratio = F(q[d]) / F(p[d]) if F(p[d]) != 0 else (F(np.inf) if F(q[d]) > 0 else F(np.nan))
    if F(ra) < ratio:
        return True, None
    adj = []
    s = F(0)
    for qi, pi in zip(q, p):
        diff = F(F(qi) - F(pi))
        diff = diff if diff >= 0 else F(0)  # Swift max(0, y)
        adj.append(diff)
        s = F(s + diff)
    if s > 0:
        adj = [F(a / s) for a in adj]
    else:
        adj = [F(x) for x in q]
    return False, sample_from_probs(adj, rr)


def verify_sequence(drafts, p, q, seed, step, seq):  # :95-129
    out = []
    k = len(drafts)
    for i in range(k):
        ok, nt = verify_token(drafts[i], p[i], q[i], uniform(seed, step, seq, i, 1), uniform(seed, step, seq, i, 2))
        if ok:
            out.append(int(drafts[i]))
        else:
            out.append(int(nt))
            return out
    out.append(sample_from_probs(q[k], uniform(seed, step, seq, k, 3)))
    return out


def f32list(a):
    return [float(F(x)) for x in a]


def main():
    kat = {"philox": [{"ctr": c, "key": k, "out": o} for c, k, o in PHILOX_KAT]}
    for c, k, o in PHILOX_KAT:
        assert philox(c, k) == o, "pure-Python Philox disagrees with the published vectors"
    kat["uniform"] = [{"coord": [s, st, sq, ps, sl], "u": uniform(s, st, sq, ps, sl)}
                      for (s, st, sq, ps, sl) in [(0, 0, 0, 0, 0), (1234, 7, 3, 2, 1), (2**40 + 5, 99, 63, 4, 3),
                                                  (42, 1, 0, 0, 2)]]
    sfp = [
        {"probs": [0.5, 0.5], "r": 0.5, "expect": 0, "why": "r <= cdf is inclusive (:68): 0.5 <= 0.5 at i=0"},
        {"probs": [0.1, 0.2], "r": 0.9, "expect": 1, "why": "cdf never reaches r: fallback V-1 (:72)"},
        {"probs": [0.0, 1.0], "r": 0.0, "expect": 0, "why": "r = 0 <= cdf = 0 picks a zero-probability index 0"},
        {"probs": [0.25, 0.25, 0.25, 0.25], "r": 0.6, "expect": 2, "why": "cdf 0.25, 0.5, 0.75 -> i = 2"},
    ]
    rng = np.random.default_rng(2024)
    for n in (7, 33, 257):
        pr = rng.random(n).astype(F)
        pr = (pr / pr.sum(dtype=np.float64)).astype(F)
        r = float(F(rng.random()))
        sfp.append({"probs": f32list(pr), "r": r, "expect": sample_from_probs(pr, r), "why": "random, restated"})
    kat["sample_from_probs"] = sfp
    vt = [
        {"d": 1, "p": [0.25] * 4, "q": [0.25] * 4, "ra": 0.999, "rr": 0.5, "accept": True,
         "why": "q = p: ratio 1, r < 1 always accepts (:32)"},
        {"d": 0, "p": [0.0, 0.5, 0.5], "q": [0.2, 0.3, 0.5], "ra": 0.99, "rr": 0.0, "accept": True,
         "why": "p[d] = 0, q[d] > 0: ratio = +inf accepts"},
        {"d": 0, "p": [0.0, 0.5, 0.5, 0.0], "q": [0.0, 0.0, 0.5, 0.5], "ra": 0.0, "rr": 0.3, "accept": False,
         "token": 3, "why": "0/0 = NaN: r < NaN is false -> reject; residual [0,0,0,0.5]/0.5 -> token 3"},
        {"d": 0, "p": [0.5, 0.5], "q": [0.25, 0.25], "ra": 0.7, "rr": 0.4, "accept": False, "token": 1,
         "why": "ratio 0.5 < r -> reject; residual sums to 0 -> falls back to q (:52-55); cdf 0.25, 0.5 -> 1"},
        {"d": 2, "p": [0.3, 0.2, 0.5], "q": [0.1, 0.6, 0.3], "ra": 0.75, "rr": 0.01, "accept": False, "token": 1,
         "why": "ratio 0.6 < 0.75 -> reject; residual mass only at 1"},
    ]
    for c in vt:
        ok, nt = verify_token(c["d"], c["p"], c["q"], c["ra"], c["rr"])
        assert ok == c["accept"] and (ok or nt == c["token"]), c["why"]
    kat["verify_token"] = vt
    seqs = []
    for case in range(16):
        V = int(rng.choice([5, 17, 64, 128]))
        k = int(rng.choice([1, 2, 4, 5]))
        p = rng.random((k, V)).astype(F) ** 3
        q = rng.random((k + 1, V)).astype(F) ** 3
        p = (p / p.sum(axis=1, keepdims=True, dtype=np.float64)).astype(F)
        q = (q / q.sum(axis=1, keepdims=True, dtype=np.float64)).astype(F)
        if case % 4 == 1:
            q[:k] = p  # identical rows: everything accepted, bonus sampled
        drafts = [int(rng.integers(V)) for _ in range(k)]
        seed, step, seq = int(rng.integers(2**63)), int(rng.integers(1000)), int(rng.integers(64))
        seqs.append({"V": V, "k": k, "p": [f32list(r) for r in p], "q": [f32list(r) for r in q], "drafts": drafts,
                     "seed": seed, "step": step, "seq": seq,
                     "expect": verify_sequence(drafts, p, q, seed, step, seq)})
    kat["verify_sequence"] = seqs
    OUT.write_text(json.dumps(kat))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
