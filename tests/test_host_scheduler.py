"""libyk_host.so's scheduling logic on the CPU: host/yk_host.cpp compiled with a
stand-in for the six device entry points it calls (tests/host_stub/yk_stub.cpp),
which checks every page table it is given.  Covers admission to completion, page
accounting, sliding-window reclamation (which must never hand a forward a page it
may still read) and the streaming callbacks.  No GPU."""
from __future__ import annotations

import ctypes as C
import shutil
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
_P = C.c_void_p
_U32P = C.POINTER(C.c_uint32)
ON_TOKENS = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, _U32P, C.c_int32)
ON_DONE = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, C.c_int32)
K, V = 4, 1000


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("g++ not found")
    out = tmp_path_factory.mktemp("hoststub") / "libyk_host_stub.so"
    # YKH_STUB_SANITIZE=1 builds with AddressSanitizer + UBSan; run pytest with
    # LD_PRELOAD=$(g++ -print-file-name=libasan.so) so the runtime loads first.
    san = ["-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=undefined"] if os.environ.get("YKH_STUB_SANITIZE") else []
    subprocess.run([cxx, "-O1", "-std=c++17", "-fPIC", "-shared", "-Wl,-Bsymbolic", *san, "-o", str(out),
                    str(ROOT / "yanaiengine_b200" / "host" / "yk_host.cpp"), str(ROOT / "tests" / "host_stub" / "yk_stub.cpp"),
                    f"-I{ROOT / 'include'}"], check=True, capture_output=True)
    L = C.CDLL(str(out))
    for name, res, args in (
        ("stub_model", _P, [C.c_int, C.c_int, C.c_int, C.c_int]), ("stub_model_free", None, [_P]),
        ("stub_pool", _P, [C.c_int]), ("stub_pool_free", None, [_P]),
        ("stub_sampler", _P, [C.c_int, C.c_int]), ("stub_sampler_free", None, [_P]),
        ("stub_stats", None, [C.POINTER(C.c_int64)] * 3), ("stub_reset", None, []),
        ("ykh_scheduler_create", C.c_int32, [_P, _P, _P, _P, _P, C.c_int32, C.c_float, C.c_uint64, C.POINTER(_P)]),
        ("ykh_scheduler_destroy", None, [_P]),
        ("ykh_submit", C.c_int32, [_P, _U32P, C.c_int32, C.c_int32, C.c_int64, C.c_uint32]),
        ("ykh_submit_cached", C.c_int32, [_P, _U32P, C.c_int32, C.c_int32, C.c_int64, C.c_uint32]),
        ("ykh_submit_stream", C.c_int32, [_P, _U32P, C.c_int32, C.c_int32, C.c_int64, C.c_uint32, C.c_void_p,
                                          C.c_void_p, C.c_void_p]),
        ("ykh_step", C.c_int32, [_P, C.POINTER(C.c_int32)]),
        ("ykh_num_running", C.c_int32, [_P]), ("ykh_num_waiting", C.c_int32, [_P]),
        ("ykh_generated", C.c_int32, [_P, C.c_uint32, _U32P, C.c_int32, C.POINTER(C.c_int32)]),
        ("ykh_usage", C.c_float, [_P, C.c_int32]),
        ("ykh_set_window_reclaim", C.c_int32, [_P, C.c_int32]),
        ("ykh_scheduler_create_split", C.c_int32, [_P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_float, C.c_uint64,
                                                   C.POINTER(_P)]),
        ("ykh_usage_windowed", C.c_float, [_P, C.c_int32]),
        ("stub_group", _P, [C.c_int]), ("stub_group_free", None, [_P]),
        ("stub_engine", _P, [_P, C.c_int]), ("stub_engine_free", None, [_P]),
        ("ykh_set_draft_shard", C.c_int32, [_P, _P, C.c_int32, C.c_int32]),
    ):
        f = getattr(L, name)
        f.restype, f.argtypes = res, args
    return L


class Rig:
    """A scheduler over stub models: target and draft share the window schedule."""

    def __init__(self, L, blocks, window=0, parity=-1, reclaim=True, wblocks=0, shard=None, dblocks=None):
        """wblocks > 0: split pools (windowed layers in pools of wblocks blocks);
        shard = (engine, rank, world): sequence-sharded drafting; dblocks: draft pool size."""
        self.L = L
        self.t = L.stub_model(4, window, parity, V)
        self.d = L.stub_model(2, window, parity, V)
        self.tp, self.dp = L.stub_pool(blocks), L.stub_pool(dblocks or blocks)
        self.twp = L.stub_pool(wblocks) if wblocks else None
        self.dwp = L.stub_pool(wblocks) if wblocks else None
        self.s = L.stub_sampler(K, V)
        self.h = _P()
        if wblocks:
            assert L.ykh_scheduler_create_split(self.t, self.tp, self.twp, self.d, self.dp, self.dwp, self.s, K, 0.8,
                                                1, C.byref(self.h)) == 0
        else:
            assert L.ykh_scheduler_create(self.t, self.tp, self.d, self.dp, self.s, K, 0.8, 1, C.byref(self.h)) == 0
        assert L.ykh_set_window_reclaim(self.h, 1 if reclaim else 0) == 0
        if shard is not None:
            assert L.ykh_set_draft_shard(self.h, *shard) == 0
        else:
            L.stub_reset()
        self.keep = []

    def submit(self, seq, n, max_tokens, stream=None, cached=False):
        p = (C.c_uint32 * n)(*[(seq * 17 + i) % V for i in range(n)])
        if cached:
            return self.L.ykh_submit_cached(self.h, p, n, max_tokens, -1, seq)
        if stream is None:
            assert self.L.ykh_submit(self.h, p, n, max_tokens, -1, seq) == 0
        else:
            ct = ON_TOKENS(lambda _u, sid, toks, m: stream[0](int(sid), [toks[i] for i in range(m)]))
            cd = ON_DONE(lambda _u, sid, m: stream[1](int(sid), int(m)))
            self.keep.append((ct, cd))
            assert self.L.ykh_submit_stream(self.h, p, n, max_tokens, -1, seq, C.cast(ct, C.c_void_p),
                                            C.cast(cd, C.c_void_p), None) == 0

    def run(self, max_steps=500):
        usage = []
        for _ in range(max_steps):
            if self.L.ykh_num_running(self.h) == 0 and self.L.ykh_num_waiting(self.h) == 0:
                return usage, 0
            e = C.c_int32()
            st = self.L.ykh_step(self.h, C.byref(e))
            if st != 0:
                return usage, st
            usage.append((self.L.ykh_usage(self.h, 0), self.L.ykh_usage_windowed(self.h, 0),
                          self.L.ykh_usage_windowed(self.h, 1)) if self.twp else self.L.ykh_usage(self.h, 0))
        return usage, -1

    def generated(self, seq):
        n = C.c_int32()
        buf = (C.c_uint32 * 4096)()
        assert self.L.ykh_generated(self.h, seq, buf, 4096, C.byref(n)) == 0
        return list(buf[: n.value])

    def stats(self):
        v, f, p = C.c_int64(), C.c_int64(), C.c_int64()
        self.L.stub_stats(C.byref(v), C.byref(f), C.byref(p))
        return v.value, f.value, p.value

    def close(self):
        self.L.ykh_scheduler_destroy(self.h)
        for x, free in ((self.t, self.L.stub_model_free), (self.d, self.L.stub_model_free),
                        (self.tp, self.L.stub_pool_free), (self.dp, self.L.stub_pool_free),
                        (self.s, self.L.stub_sampler_free)):
            free(x)
        for x in (self.twp, self.dwp):
            if x:
                self.L.stub_pool_free(x)


def test_batch_runs_to_completion(lib):
    r = Rig(lib, blocks=256)
    try:
        for i in range(5):
            r.submit(i, 10 + 13 * i, max_tokens=30)
        usage, st = r.run()
        assert st == 0
        viol, fwd, pages = r.stats()
        assert viol == 0 and fwd > 0 and pages > 0
        for i in range(5):
            assert 30 <= len(r.generated(i)) <= 30 + K
        assert usage[-1] == 0.0  # every page back in the free list
    finally:
        r.close()


def test_window_reclamation_bounds_memory_and_keeps_reads_valid(lib):
    """Every layer windowed (24 tokens): 4 sequences of 30 + 200 tokens need ~60
    pages each model without reclamation but fit in 40 with it; no forward is ever
    handed a freed (or shared) page inside its window."""
    off = Rig(lib, blocks=40, window=24, parity=-1, reclaim=False)
    try:
        for i in range(4):
            off.submit(i, 30, max_tokens=200)
        _, st = off.run()
        assert st == 2  # YK_ERR_OOM: the pages of every past token are kept
    finally:
        off.close()
    on = Rig(lib, blocks=40, window=24, parity=-1, reclaim=True)
    try:
        for i in range(4):
            on.submit(i, 30, max_tokens=200)
        usage, st = on.run()
        assert st == 0
        viol, fwd, pages = on.stats()
        assert viol == 0 and pages > 0
        assert max(usage) <= 4 * 4 / 40 + 1e-6  # at most ~4 live pages per sequence
        assert all(len(on.generated(i)) >= 200 for i in range(4))
        assert usage[-1] == 0.0
    finally:
        on.close()


def test_alternating_windows_free_nothing(lib):
    """Gemma's schedule (windowed on even layers only): a page holds every layer,
    the global layers still read it, so nothing is reclaimed."""
    a = Rig(lib, blocks=256, window=24, parity=0, reclaim=True)
    b = Rig(lib, blocks=256, window=0, parity=-1, reclaim=True)
    try:
        for r in (a, b):
            for i in range(3):
                r.submit(i, 40, max_tokens=60)
        ua, sa = a.run()
        ub, sb = b.run()
        assert sa == 0 and sb == 0 and ua == ub
        assert a.stats()[0] == 0
    finally:
        a.close()
        b.close()


def test_streaming_runs_concatenate_to_generated(lib):
    r = Rig(lib, blocks=256)
    runs, done = {}, {}
    cb = (lambda sid, toks: runs.setdefault(sid, []).append(toks), lambda sid, n: done.setdefault(sid, []).append(n))
    try:
        for i in range(3):
            r.submit(i, 20 + 5 * i, max_tokens=25, stream=cb)
        r.submit(7, 15, max_tokens=25)
        _, st = r.run()
        assert st == 0
        for i in range(3):
            g = r.generated(i)
            assert [x for run in runs[i] for x in run] == g
            assert all(1 <= len(run) <= K + 1 for run in runs[i])
            assert done[i] == [len(g)]
        assert 7 not in runs and 7 not in done
    finally:
        r.close()


def test_deterministic(lib):
    outs = []
    for _ in range(2):
        r = Rig(lib, blocks=128, window=24, parity=-1)
        try:
            for i in range(3):
                r.submit(i, 33, max_tokens=50)
            _, st = r.run()
            assert st == 0
            outs.append([r.generated(i) for i in range(3)])
        finally:
            r.close()
    assert outs[0] == outs[1]


def test_stub_catches_bad_tables(lib):
    """The stand-in's page-table check itself: a block read by two sequences, or one outside the pool,
    counts as a violation (a planted mistake, on the CPU stand-in)."""
    f = lib.yk_forward_step
    f.restype = C.c_int32
    f.argtypes = [_P, _P, _U32P, C.c_int32, _U32P, _U32P, C.c_int32, C.POINTER(C.c_int32), C.c_int32, C.c_int32,
                  C.POINTER(C.c_int32)]
    r = Rig(lib, blocks=8)
    try:
        toks = (C.c_uint32 * 2)(1, 2)
        qs = (C.c_uint32 * 3)(0, 1, 2)
        ctx = (C.c_uint32 * 2)(20, 20)  # two pages each
        rows = C.c_int32()
        ok = (C.c_int32 * 4)(0, 1, 2, 3)
        assert f(r.t, r.tp, toks, 2, qs, ctx, 2, ok, 2, 0, C.byref(rows)) == 0
        assert r.stats()[0] == 0
        shared = (C.c_int32 * 4)(0, 1, 2, 1)  # block 1 in both sequences' windows
        f(r.t, r.tp, toks, 2, qs, ctx, 2, shared, 2, 0, C.byref(rows))
        assert r.stats()[0] == 1
        outside = (C.c_int32 * 4)(0, 1, 2, 9)  # block 9 of an 8-block pool
        f(r.t, r.tp, toks, 2, qs, ctx, 2, outside, 2, 0, C.byref(rows))
        assert r.stats()[0] == 2
    finally:
        r.close()


def test_split_pools_free_windowed_pages(lib):
    """Gemma's schedule (windowed on even layers) over split pools: the windowed
    layers' pool stays at a few pages per sequence while the global layers' pool
    keeps every page; every table each forward gets is valid for its reads."""
    r = Rig(lib, blocks=256, window=24, parity=0, reclaim=True, wblocks=24)
    try:
        for i in range(4):
            r.submit(i, 30, max_tokens=150)
        usage, st = r.run()
        assert st == 0
        viol, fwd, pages = r.stats()
        assert viol == 0 and pages > 0
        assert max(u[1] for u in usage) <= 4 * 4 / 24 + 1e-6 and max(u[2] for u in usage) <= 4 * 4 / 24 + 1e-6
        assert max(u[0] for u in usage) > 4 * 10 / 256  # the global layers keep their pages
        assert usage[-1] == (0.0, 0.0, 0.0)
        keep = Rig(lib, blocks=256, window=24, parity=0, reclaim=True)
        try:
            for i in range(4):
                keep.submit(i, 30, max_tokens=150)
            assert keep.run()[1] == 0
            assert [r.generated(i) for i in range(4)] == [keep.generated(i) for i in range(4)]
        finally:
            keep.close()
        # without reclamation the 24-block windowed pools run out
        off = Rig(lib, blocks=256, window=24, parity=0, reclaim=False, wblocks=24)
        try:
            for i in range(4):
                off.submit(i, 30, max_tokens=150)
            assert off.run()[1] == 2
        finally:
            off.close()
    finally:
        r.close()


def test_cached_prompts_longer_than_the_window_over_split_pools(lib):
    """Prompts already in the cache (the benchmark's synthetic contexts), longer
    than the window, over split pools with reclamation: the windowed pools take
    only the pages inside the window at admission (a windowed pool far smaller
    than the prompts suffices), every table a forward gets is valid, and the
    tokens equal those of the same run over one pool per model."""
    r = Rig(lib, blocks=256, window=24, parity=0, reclaim=True, wblocks=16)
    try:
        for i in range(4):
            assert r.submit(i, 90 + 7 * i, max_tokens=40, cached=True) == 0
        usage, st = r.run()
        assert st == 0
        viol, fwd, pages = r.stats()
        assert viol == 0 and fwd > 0
        keep = Rig(lib, blocks=256, window=24, parity=0, reclaim=True)
        try:
            for i in range(4):
                assert keep.submit(i, 90 + 7 * i, max_tokens=40, cached=True) == 0
            assert keep.run()[1] == 0
            assert [r.generated(i) for i in range(4)] == [keep.generated(i) for i in range(4)]
        finally:
            keep.close()
        # without reclamation the 16-block windowed pools cannot hold the prompts
        off = Rig(lib, blocks=256, window=24, parity=0, reclaim=False, wblocks=16)
        try:
            got = [off.submit(i, 90 + 7 * i, max_tokens=40, cached=True) for i in range(4)]
            assert got[:2] == [0, 0] and 2 in got  # YK_ERR_OOM once the 16 blocks are used
        finally:
            off.close()
    finally:
        r.close()


def test_sharded_drafting_matches_one_rank(lib):
    """Sequence-sharded drafting (tensor parallelism: every rank runs the scheduler
    over the whole batch, drafts and verifies only its slice, all-gathers drafts and
    results): ranks emulated as threads of one process with a rendezvous all-gather.
    Every rank's tokens equal a single-rank run's; each rank's draft pool only needs
    room for its slice; slices move when sequences finish at different times."""
    import threading

    reqs = [(i, 20 + 9 * i, 12 + 7 * (i % 4)) for i in range(7)]  # (seq, prompt length, max_tokens)
    for cached in (False, True):
        _sharded_case(lib, reqs, cached)


def _sharded_case(lib, reqs, cached):
    import threading

    ref = Rig(lib, blocks=256)
    try:
        for sid, n, mt in reqs:
            assert ref.submit(sid, n, max_tokens=mt, cached=cached) in (None, 0)
        assert ref.run()[1] == 0
        want = [ref.generated(sid) for sid, _, _ in reqs]
    finally:
        ref.close()
    for world, dblocks in ((2, 24), (3, 16)):
        # a draft pool with room for about one slice of the batch: too small for all of it
        small = Rig(lib, blocks=256, dblocks=dblocks)
        try:
            st = [small.submit(sid, n, max_tokens=mt, cached=cached) for sid, n, mt in reqs]
            assert 2 in st or small.run()[1] == 2  # YK_ERR_OOM without sharding
        finally:
            small.close()
        lib.stub_reset()
        g = lib.stub_group(world)
        engines = [lib.stub_engine(g, r) for r in range(world)]
        rigs = [Rig(lib, blocks=256, shard=(engines[r], r, world), dblocks=dblocks) for r in range(world)]
        status = [None] * world
        try:
            for rig in rigs:
                for sid, n, mt in reqs:
                    assert rig.submit(sid, n, max_tokens=mt, cached=cached) in (None, 0)

            def run(r):
                status[r] = rigs[r].run()[1]

            th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
            for t in th:
                t.start()
            for t in th:
                t.join(timeout=60)
            assert not any(t.is_alive() for t in th)
            assert status == [0] * world
            for rig in rigs:
                assert [rig.generated(sid) for sid, _, _ in reqs] == want
            viol, fwd, _ = rigs[0].stats()
            assert viol == 0 and fwd > 0
        finally:
            for rig in rigs:
                rig.close()
            for e in engines:
                lib.stub_engine_free(e)
            lib.stub_group_free(g)


from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.lists(st.tuples(st.integers(1, 70), st.integers(1, 60)), min_size=1, max_size=6),
       st.sampled_from([(0, -1), (16, -1), (24, -1), (24, 0), (40, 1)]), st.booleans(), st.booleans(),
       st.integers(24, 160))
def test_scheduler_property(lib, reqs, schedule, reclaim, split, blocks):
    """Random batches, window schedules, pool sizes, reclamation on/off, one or two
    pools: a run either completes -- every request with at least max_tokens tokens,
    every page returned, no forward ever handed an invalid or shared page -- or
    stops with YK_ERR_OOM; it never corrupts the page tables."""
    window, parity = schedule
    split = split and window > 0 and parity >= 0  # split pools need global and windowed layers
    r = Rig(lib, blocks=blocks, window=window, parity=parity, reclaim=reclaim, wblocks=blocks if split else 0)
    try:
        for i, (n, mt) in enumerate(reqs):
            r.submit(i, n, max_tokens=mt)
        usage, st_ = r.run(max_steps=400)
        assert st_ in (0, 2), st_
        assert r.stats()[0] == 0
        if st_ == 0:
            for i, (_, mt) in enumerate(reqs):
                assert mt <= len(r.generated(i)) <= mt + K
            last = usage[-1] if usage else 0.0
            assert (last == (0.0, 0.0, 0.0)) if split else (last == 0.0)
    finally:
        r.close()
