"""End-to-end draft->verify through libyk_host.so's Scheduler vs the oracle.

The small fp32 speculative workload (d=2048 target + d=512 draft, batch 1, k=4, greedy,
prompt of 128 uniform ids, 16-token pages): the emitted tokens must be
identical to the oracle's speculative run, and -- the defining property of
greedy speculative decoding -- identical to plain greedy decoding of the target.
"""
import os

import numpy as np
import pytest

from helpers import SMALL_F32_DRAFT, SMALL_F32_TARGET, TINY, PageTables, gpu_model, oracle_twin, step_inputs
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu
NTHREADS = max(4, os.cpu_count() or 4)


def oracle_greedy_spec(orc_t, orc_d, prompt, k, steps, runs=None):
    """Restates ykh_step for one sequence with greedy draft sampling and verification
    (runs, if given, receives each step's emitted run)."""
    pt_t, pt_d = PageTables(orc_t.num_blocks), PageTables(orc_d.num_blocks)
    tokens = list(prompt)
    tpos = dpos = 0
    for _ in range(steps):
        N = len(tokens)
        drafts = []
        for j in range(k):
            inp = tokens[dpos:N] if j == 0 else [drafts[-1]]
            lg = orc_d.forward(*step_inputs(pt_d, [(0, inp, dpos)]), last_n=1)
            dpos += len(inp)
            drafts.append(int(np.argmax(lg[-1])))
        inp = tokens[tpos:N] + drafts
        lg = orc_t.forward(*step_inputs(pt_t, [(0, inp, tpos)]), last_n=k + 1)
        out = []
        for i in range(k):
            a = int(np.argmax(lg[i]))
            out.append(a)
            if a != drafts[i]:
                break
        else:
            out.append(int(np.argmax(lg[k])))
        acc = len(out) - 1
        tpos = N + acc
        dpos = min(dpos, N + acc)
        tokens += out
        if runs is not None:
            runs.append(out)
    return tokens[len(prompt):]


def oracle_greedy_plain(orc_t, prompt, n_new):
    pt = PageTables(orc_t.num_blocks)
    tokens = list(prompt)
    pos = 0
    while len(tokens) < len(prompt) + n_new:
        lg = orc_t.forward(*step_inputs(pt, [(0, tokens[pos:], pos)]), last_n=1)
        pos = len(tokens)
        tokens.append(int(np.argmax(lg[-1])))
    return tokens[len(prompt):]


def _run(engine, oracle, tcfg, dcfg, dtype, prompt_len, k, steps, seed_t, seed_d, nb=64):
    t, tp = gpu_model(engine, tcfg, dtype, seed=seed_t, num_blocks=nb, max_tokens=prompt_len + 8, max_seqs=4)
    d, dp = gpu_model(engine, dcfg, dtype, seed=seed_d, num_blocks=nb, max_tokens=prompt_len + 8, max_seqs=4)
    s = abi.Sampler(engine, 4, k, tcfg["vocab_size"])
    sch = abi.Scheduler(t, tp, d, dp, s, k, 0.0, 77)
    try:
        prompt = np.random.default_rng(128).integers(0, tcfg["vocab_size"], prompt_len).tolist()
        sch.submit(prompt, max_tokens=10**6, stop_token=-1, seq_id=0)
        for _ in range(steps):
            sch.step()
        got = sch.generated(0)
        orc_t = oracle_twin(oracle, t, tcfg, nb, emulate_bf16=False, nthreads=NTHREADS)
        orc_d = oracle_twin(oracle, d, dcfg, nb, emulate_bf16=False, nthreads=NTHREADS)
        return got, orc_t, orc_d, prompt
    finally:
        sch.close()
        s.close()
        dp.close()
        d.close()
        tp.close()
        t.close()


def test_small_f32_greedy_token_identical(engine, oracle):
    got, orc_t, orc_d, prompt = _run(engine, oracle, SMALL_F32_TARGET, SMALL_F32_DRAFT, abi.DTYPE_F32, 128, 4, 5, 1, 2)
    ref = oracle_greedy_spec(orc_t, orc_d, prompt, 4, 5)
    assert got == ref
    # greedy speculative decoding == greedy decoding of the target alone
    assert got == oracle_greedy_plain(orc_t, prompt, len(got))


def test_tiny_greedy_spec_equals_plain_greedy(engine, oracle):
    """Same property with a draft that disagrees often (different seed): many rejections."""
    got, orc_t, orc_d, prompt = _run(engine, oracle, TINY, dict(TINY, n_layers=1), abi.DTYPE_F32, 40, 4, 12, 5, 9)
    assert len(got) >= 12
    assert got == oracle_greedy_spec(orc_t, orc_d, prompt, 4, 12)
    assert got == oracle_greedy_plain(orc_t, prompt, len(got))


def test_scheduler_sampled_batch_runs(engine):
    """T > 0, several sequences of different lengths, stop on max_tokens, pages returned."""
    t, tp = gpu_model(engine, TINY, abi.DTYPE_BF16, seed=1, num_blocks=128, max_tokens=256, max_seqs=8)
    d, dp = gpu_model(engine, dict(TINY, n_layers=1), abi.DTYPE_BF16, seed=2, num_blocks=128, max_tokens=256,
                      max_seqs=8)
    s = abi.Sampler(engine, 8, 5, TINY["vocab_size"])
    sch = abi.Scheduler(t, tp, d, dp, s, 5, 0.8, 3)
    try:
        rng = np.random.default_rng(0)
        for i in range(6):
            sch.submit(rng.integers(0, 512, 10 + 7 * i).tolist(), max_tokens=20, stop_token=-1, seq_id=i)
        total = 0
        for _ in range(30):
            if sch.running() == 0 and sch.waiting() == 0:
                break
            total += sch.step()
        assert sch.running() == 0 and sch.waiting() == 0
        steps, emitted, accepted = sch.counters()
        assert emitted == total and emitted >= 6 * 20
        for i in range(6):
            g = sch.generated(i)
            assert 20 <= len(g) <= 25 and all(0 <= x < 512 for x in g)
        assert sch.usage() == 0.0 and sch.usage(draft=True) == 0.0
    finally:
        sch.close()
        s.close()
        dp.close()
        d.close()
        tp.close()
        t.close()


def test_scheduler_streaming_callbacks(engine):
    """ykh_submit_stream (the server's onTokenGenerated / onCompletion): every
    step's emitted run arrives in order, the runs concatenate to the generated
    list, completion fires once per request (stop token or max_tokens), and plain
    and streaming requests share a batch."""
    t, tp = gpu_model(engine, TINY, abi.DTYPE_BF16, seed=1, num_blocks=128, max_tokens=256, max_seqs=8)
    d, dp = gpu_model(engine, dict(TINY, n_layers=1), abi.DTYPE_BF16, seed=2, num_blocks=128, max_tokens=256,
                      max_seqs=8)
    s = abi.Sampler(engine, 8, 4, TINY["vocab_size"])
    sch = abi.Scheduler(t, tp, d, dp, s, 4, 0.8, 5)
    runs, done = {}, {}
    try:
        rng = np.random.default_rng(1)
        for i in range(4):
            sch.submit_stream(rng.integers(0, 512, 12 + 5 * i).tolist(), max_tokens=15,
                              on_tokens=lambda sid, toks: runs.setdefault(sid, []).append(toks),
                              on_done=lambda sid, n: done.setdefault(sid, []).append(n), seq_id=i)
        sch.submit(rng.integers(0, 512, 9).tolist(), max_tokens=15, stop_token=-1, seq_id=9)
        for _ in range(40):
            if sch.running() == 0 and sch.waiting() == 0:
                break
            sch.step()
        assert sch.running() == 0 and sch.waiting() == 0
        for i in range(4):
            g = sch.generated(i)
            assert [x for run in runs[i] for x in run] == g
            assert all(1 <= len(run) <= 5 for run in runs[i])  # at most k + 1 tokens per step
            assert done[i] == [len(g)] and len(g) >= 15
        assert 9 not in runs and 9 not in done and len(sch.generated(9)) >= 15
    finally:
        sch.close()
        s.close()
        dp.close()
        d.close()
        tp.close()
        t.close()


def test_streaming_matches_oracle_spec_run(engine, oracle):
    """The server path (S/InferenceServer.swift:118-126,167-176: onTokenGenerated per
    token, onCompletion once) through ykh_submit_stream on the tiny fp32 greedy
    pair with many rejections: every streamed run equals the oracle's speculative
    step run, in order, and completion reports the generated count once."""
    k, max_tokens = 4, 30
    tcfg, dcfg = TINY, dict(TINY, n_layers=1)
    t, tp = gpu_model(engine, tcfg, abi.DTYPE_F32, seed=5, num_blocks=64, max_tokens=48, max_seqs=4)
    d, dp = gpu_model(engine, dcfg, abi.DTYPE_F32, seed=9, num_blocks=64, max_tokens=48, max_seqs=4)
    s = abi.Sampler(engine, 4, k, tcfg["vocab_size"])
    sch = abi.Scheduler(t, tp, d, dp, s, k, 0.0, 77)
    runs, done = [], []
    try:
        prompt = np.random.default_rng(128).integers(0, tcfg["vocab_size"], 40).tolist()
        sch.submit_stream(prompt, max_tokens=max_tokens, on_tokens=lambda sid, toks: runs.append((sid, toks)),
                          on_done=lambda sid, n: done.append((sid, n)), seq_id=3)
        for _ in range(max_tokens + 2):
            if sch.running() == 0 and sch.waiting() == 0:
                break
            sch.step()
        assert sch.running() == 0 and sch.waiting() == 0
        orc_t = oracle_twin(oracle, t, tcfg, 64, emulate_bf16=False, nthreads=NTHREADS)
        orc_d = oracle_twin(oracle, d, dcfg, 64, emulate_bf16=False, nthreads=NTHREADS)
        ref_runs = []
        oracle_greedy_spec(orc_t, orc_d, prompt, k, len(runs), ref_runs)
        assert [sid for sid, _ in runs] == [3] * len(runs)
        assert [toks for _, toks in runs] == ref_runs
        streamed = [x for _, toks in runs for x in toks]
        assert len(streamed) >= max_tokens and streamed == sch.generated(3)
        assert done == [(3, len(streamed))]
    finally:
        sch.close()
        s.close()
        dp.close()
        d.close()
        tp.close()
        t.close()


def test_window_block_reclamation(engine):
    """Every layer windowed (width 24): with reclamation the pages wholly before the
    window go back to the allocator and are reused by the other sequence, and the
    greedy tokens are identical to a run that keeps every page (no freed page is
    ever read again)."""
    cfg = dict(TINY, window=24, window_layer_parity=-1)
    t, tp = gpu_model(engine, cfg, abi.DTYPE_BF16, seed=1, num_blocks=64, max_tokens=256, max_seqs=8)
    d, dp = gpu_model(engine, dict(cfg, n_layers=1), abi.DTYPE_BF16, seed=2, num_blocks=64, max_tokens=256,
                      max_seqs=8)
    s = abi.Sampler(engine, 8, 4, TINY["vocab_size"])
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 512, n).tolist() for n in (40, 55)]

    def run(reclaim):
        sch = abi.Scheduler(t, tp, d, dp, s, 4, 0.0, 7)
        try:
            sch.set_window_reclaim(reclaim)
            for i, pr in enumerate(prompts):
                sch.submit(pr, max_tokens=80, stop_token=-1, seq_id=i)
            usage = []
            for _ in range(200):
                if sch.running() == 0 and sch.waiting() == 0:
                    break
                sch.step()
                usage.append((sch.usage(), sch.usage(draft=True)))
            assert sch.running() == 0 and sch.waiting() == 0
            return [sch.generated(i) for i in range(2)], usage
        finally:
            sch.close()

    try:
        keep, u_keep = run(False)
        free, u_free = run(True)
        assert keep == free
        assert all(len(g) >= 80 for g in free)
        n = min(len(u_keep), len(u_free))
        # kept: all 17 pages of the two sequences at the end; reclaimed: the window's 2-3 pages
        # plus the step's new tokens per sequence
        assert max(u[0] for u in u_free[:n]) < 0.6 * max(u[0] for u in u_keep[:n])
        assert max(u[1] for u in u_free[:n]) < 0.6 * max(u[1] for u in u_keep[:n])
        assert u_free[-1] == (0.0, 0.0)
        assert engine.device_error() == 0
    finally:
        s.close()
        dp.close()
        d.close()
        tp.close()
        t.close()


def test_split_pools_reclaim_windowed_pages(engine):
    """Alternating windows (even layers, width 24) over split pools with
    reclamation: greedy tokens identical to single pools that keep every page,
    and the windowed pools stay small."""
    cfg = dict(TINY, window=24, window_layer_parity=0)
    dcfg = dict(cfg, n_layers=2)
    mk = lambda c, seed: abi.Model(engine, abi.make_config(**c, dtype=abi.DTYPE_BF16, max_tokens=256, max_seqs=8),
                                   seed=seed, init_std=0.02)
    t, d = mk(cfg, 1), mk(dcfg, 2)
    s = abi.Sampler(engine, 8, 4, TINY["vocab_size"])
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 512, n).tolist() for n in (40, 55)]
    pools = []

    def pool(m, layers):
        pools.append(abi.KVPool(engine, m.cfg, 64, layers))
        return pools[-1]

    def run(split):
        if split:
            sch = abi.Scheduler(t, pool(t, abi.POOL_GLOBAL_LAYERS), d, pool(d, abi.POOL_GLOBAL_LAYERS), s, 4, 0.0, 7,
                                twpool=pool(t, abi.POOL_WINDOWED_LAYERS), dwpool=pool(d, abi.POOL_WINDOWED_LAYERS))
        else:
            sch = abi.Scheduler(t, pool(t, abi.POOL_ALL_LAYERS), d, pool(d, abi.POOL_ALL_LAYERS), s, 4, 0.0, 7)
        try:
            for i, pr in enumerate(prompts):
                sch.submit(pr, max_tokens=80, stop_token=-1, seq_id=i)
            wmax = 0.0
            for _ in range(200):
                if sch.running() == 0 and sch.waiting() == 0:
                    break
                sch.step()
                wmax = max(wmax, sch.usage_windowed())
            assert sch.running() == 0 and sch.waiting() == 0
            return [sch.generated(i) for i in range(2)], wmax
        finally:
            sch.close()

    try:
        single, _ = run(False)
        split, wmax = run(True)
        assert single == split
        assert all(len(g) >= 80 for g in split)
        assert 0.0 < wmax <= 2 * 4 / 64 + 1e-6  # a few live pages per sequence
        assert engine.device_error() == 0
    finally:
        for p in pools:
            p.close()
        s.close()
        d.close()
        t.close()
