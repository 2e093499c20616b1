"""Tensor-parallel target (the 70B-shape path): two ranks, one GPU each, NCCL
all-reduce after o_proj and down_proj.  Each rank loads its slice of one full
set of weights; the logits of both ranks must be identical (replicated LM head
on the all-reduced stream) and must match the bf16-emulating oracle forward of
the full model: max |dlogit| <= 2e-2 * max |logit|, as for the 1-GPU forward,
with the all-reduce payload in bf16 (the default) and in fp32.  Needs two GPUs
(skipped otherwise).

The all-reduce is the group's own two-shot kernel over NVLink peer memory by
default (bf16 payload) and NCCL's otherwise; both are checked against the oracle.

Failure handling (no GPU is faulted): a group whose second rank never joins
ends set-up with YK_ERR_TIMEOUT on one GPU; on two GPUs, a rank that leaves
between steps makes the other rank's next step end with YK_ERR_TIMEOUT (its
collective cannot finish; the bounded wait aborts the communicator).  NVLS is
off in every test here."""
import os

import numpy as np
import pytest

from helpers import TINY, PageTables, step_inputs
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu
CFG = dict(TINY, n_heads=8, n_kv_heads=2, ffn_dim=384)  # TP2: 4 query heads, 1 KV head, 192 FFN columns per rank
NB = 64
WORLD = 2


def _bf16(x):
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def _full_weights(cfg, seed=3):
    rng = np.random.default_rng(seed)
    d, V, F, dh = cfg["d_model"], cfg["vocab_size"], cfg["ffn_dim"], cfg["head_dim"]
    qd, kvd, L = cfg["n_heads"] * dh, cfg["n_kv_heads"] * dh, cfg["n_layers"]
    n = lambda *s: _bf16(rng.normal(0, 0.02, s))
    w = dict(embed=n(V, d), lm_head=n(V, d), final_norm=rng.uniform(0.8, 1.2, d).astype(np.float32))
    for name, shape in (("wq", (qd, d)), ("wk", (kvd, d)), ("wv", (kvd, d)), ("wo", (d, qd)), ("wg", (F, d)),
                        ("wu", (F, d)), ("wd", (d, F))):
        w[name] = [n(*shape) for _ in range(L)]
    for name in ("n1", "n2"):
        w[name] = [rng.uniform(0.8, 1.2, d).astype(np.float32) for _ in range(L)]
    return w


def _steps(seed=1):
    rng = np.random.default_rng(seed)
    V = CFG["vocab_size"]
    steps = [[(0, rng.integers(0, V, 17).tolist(), 0), (1, rng.integers(0, V, 40).tolist(), 0),
              (2, rng.integers(0, V, 5).tolist(), 0)]]
    lens = {0: 17, 1: 40, 2: 5}
    for _ in range(2):
        s = []
        for sid in (0, 1, 2):
            s.append((sid, rng.integers(0, V, 5).tolist(), lens[sid]))
            lens[sid] += 5
        steps.append(s)
    return steps


def _load_full(m, w):
    """Every tensor through yk_model_load_tensor as the FULL tensor (bf16 words,
    fp32 norms); the shard takes its window.  o_proj and down_proj arrive in the
    reference's [in x out] layout, so the transposed window is covered too."""
    def words(x):
        return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)

    m.load(abi.T_EMBED, 0, words(w["embed"]), abi.DTYPE_BF16)
    m.load(abi.T_LM_HEAD, 0, words(w["lm_head"]), abi.DTYPE_BF16)
    m.load(abi.T_FINAL_NORM, 0, w["final_norm"], abi.DTYPE_F32)
    for l in range(CFG["n_layers"]):
        for t, name in ((abi.T_WQ, "wq"), (abi.T_WK, "wk"), (abi.T_WV, "wv"), (abi.T_WGATE, "wg"),
                        (abi.T_WUP, "wu")):
            m.load(t, l, words(w[name][l]), abi.DTYPE_BF16)
        for t, name in ((abi.T_WO, "wo"), (abi.T_WDOWN, "wd")):
            m.load(t, l, np.ascontiguousarray(words(w[name][l]).T), abi.DTYPE_BF16, abi.LAYOUT_IN_OUT)
        m.load(abi.T_NORM1, l, w["n1"][l], abi.DTYPE_F32)
        m.load(abi.T_NORM2, l, w["n2"][l], abi.DTYPE_F32)


def _worker(rank, uid, q, via_loader=False, payload="bf16", ar="own"):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["YK_TP_PAYLOAD"] = payload
    os.environ["YK_TP_AR"] = ar
    try:
        e = abi.Engine(rank)
        e.tp_init(uid, rank, WORLD)
        c = abi.make_config(**CFG, dtype=abi.DTYPE_BF16, max_tokens=128, max_seqs=8)
        m = abi.Model(e, c, seed=3, tp=(rank, WORLD))
        w = _full_weights(CFG)
        if via_loader:
            _load_full(m, w)
        dh, F = CFG["head_dim"], CFG["ffn_dim"]
        hq, hk, fl = CFG["n_heads"] // WORLD * dh, CFG["n_kv_heads"] // WORLD * dh, F // WORLD
        shard = {}
        if via_loader:  # read back what the windows loaded, for the comparison below
            for t in (abi.T_WQ, abi.T_WO, abi.T_WDOWN):
                shard[t] = m.get(t, 1)
        m.set(abi.T_EMBED, 0, w["embed"])
        m.set(abi.T_LM_HEAD, 0, w["lm_head"])
        m.set(abi.T_FINAL_NORM, 0, w["final_norm"])
        for l in range(CFG["n_layers"]):
            m.set(abi.T_WQ, l, w["wq"][l][rank * hq:(rank + 1) * hq])
            m.set(abi.T_WK, l, w["wk"][l][rank * hk:(rank + 1) * hk])
            m.set(abi.T_WV, l, w["wv"][l][rank * hk:(rank + 1) * hk])
            m.set(abi.T_WO, l, np.ascontiguousarray(w["wo"][l][:, rank * hq:(rank + 1) * hq]))
            m.set(abi.T_WGATE, l, w["wg"][l][rank * fl:(rank + 1) * fl])
            m.set(abi.T_WUP, l, w["wu"][l][rank * fl:(rank + 1) * fl])
            m.set(abi.T_WDOWN, l, np.ascontiguousarray(w["wd"][l][:, rank * fl:(rank + 1) * fl]))
            m.set(abi.T_NORM1, l, w["n1"][l])
            m.set(abi.T_NORM2, l, w["n2"][l])
        for t, got in shard.items():  # the loader's windows equal the per-shard uploads
            assert np.array_equal(got, m.get(t, 1)), f"tensor {t} window differs"
        pool = abi.KVPool(e, m.cfg, NB)
        pt = PageTables(NB)
        out = []
        for i, batch in enumerate(_steps()):
            toks, qs, ctx, bt = step_inputs(pt, batch)
            rows = m.forward(pool, toks, qs, ctx, bt, 0 if i == 0 else 5)
            out.append(m.logits(0, rows))
        err = e.device_error()
        pool.close()
        m.close()
        e.close()
        q.put((rank, out, err, None))
    except Exception as ex:  # reported to the parent, which fails the test
        q.put((rank, None, None, repr(ex)))


@pytest.mark.parametrize("via_loader,payload,ar", [(False, "bf16", "own"), (True, "bf16", "own"),
                                                    (False, "bf16", "twoshot"), (False, "bf16", "nccl"),
                                                    (False, "f32", "nccl")])
def test_tp2_forward_matches_oracle(oracle, via_loader, payload, ar):
    """ar: the all-reduce after o_proj / down_proj, the group's own kernel over NVLink
    peer memory (bf16, the default: one shot at two ranks; "twoshot": the two-phase
    form every message size above the one-shot bound takes) or NCCL's."""
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    uid = abi.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, uid, q, via_loader, payload, ar)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, out, err, exc = q.get(timeout=240)
            res[rank] = (out, err, exc)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in range(WORLD):
        assert res[rank][2] is None, res[rank][2]
        assert res[rank][1] == 0
    # the oracle forward of the full model on the same steps
    w = _full_weights(CFG)
    orc = oracle.OracleModel(CFG, w, NB, emulate_bf16=True, nthreads=8)
    pt = PageTables(NB)
    for i, batch in enumerate(_steps()):
        toks, qs, cl, bt = step_inputs(pt, batch)
        o = orc.forward(toks, qs, cl, bt, 0 if i == 0 else 5)
        g0, g1 = res[0][0][i], res[1][0][i]
        np.testing.assert_array_equal(g0, g1)  # both ranks hold the same all-reduced stream
        err = np.abs(g0 - o).max() / np.abs(o).max()
        print(f"payload {payload} ({ar} all-reduce) step {i}: max |dlogit| / max |logit| = {err:.3e}")
        assert err < 2e-2, f"step {i}: rel err {err:.3e}"


def _init_alone(q):
    """Rank 0 of a group of two whose rank 1 never calls init."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        e = abi.Engine(0)
        try:
            e.tp_init(abi.tp_unique_id(), 0, 2, timeout_ms=3000)
            q.put(("joined", None))
        except abi.YKError as ex:
            # the engine stays usable after the aborted set-up
            e.sync()
            q.put((ex.status, abi.last_error()))
        e.close()
    except Exception as ex:
        q.put(("error", repr(ex)))


def test_tp_init_times_out_when_a_rank_never_joins():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_init_alone, args=(q,))
    p.start()
    try:
        status, msg = q.get(timeout=120)
    finally:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert status == abi.YK_ERR_TIMEOUT, (status, msg)
    assert "not every rank joined" in msg


def _leaver(rank, uid, q):
    """Both ranks run one forward step; rank 1 then leaves (between steps, nothing
    in flight) and rank 0 runs a second step whose all-reduce cannot finish.  NCCL's
    all-reduce: the group's own kernel reads and writes the peers' memory, which a
    rank that exits releases."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["YK_TP_AR"] = "nccl"
    try:
        e = abi.Engine(rank)
        e.tp_init(uid, rank, WORLD, timeout_ms=8000)
        c = abi.make_config(**CFG, dtype=abi.DTYPE_BF16, max_tokens=128, max_seqs=8)
        m = abi.Model(e, c, seed=3, tp=(rank, WORLD))
        pool = abi.KVPool(e, m.cfg, NB)
        pt = PageTables(NB)
        steps = _steps()
        toks, qs, ctx, bt = step_inputs(pt, steps[0])
        m.forward(pool, toks, qs, ctx, bt, 0)
        e.sync()
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # the message is out before the process goes
            os._exit(0)  # leaves without tearing the group down, as a crashed rank would
        toks, qs, ctx, bt = step_inputs(pt, steps[1])
        try:
            m.forward(pool, toks, qs, ctx, bt, 5)
            e.sync()
            q.put((rank, "finished"))
        except abi.YKError as ex:
            q.put((rank, ex.status))
    except Exception as ex:
        q.put((rank, repr(ex)))


def test_tp_peer_leaving_ends_the_next_step_with_timeout():
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    uid = abi.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_leaver, args=(r, uid, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, what = q.get(timeout=180)
            res[rank] = what
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[1] == "left"
    assert res[0] == abi.YK_ERR_TIMEOUT, res[0]


def _spec_worker(rank, uid, q, shard):
    """The speculative scheduler over a tensor-parallel fp32 target (this rank's
    shard) and a replicated fp32 draft; shard: each rank drafts its slice."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        e = abi.Engine(rank)
        e.tp_init(uid, rank, WORLD, timeout_ms=120000)
        tc = abi.make_config(**CFG, dtype=abi.DTYPE_F32, max_tokens=256, max_seqs=8)
        dcfg = dict(CFG, n_layers=1)
        dc = abi.make_config(**dcfg, dtype=abi.DTYPE_F32, max_tokens=256, max_seqs=8)
        t = abi.Model(e, tc, seed=3, tp=(rank, WORLD))
        d = abi.Model(e, dc, seed=9)
        tpool, dpool = abi.KVPool(e, t.cfg, 128), abi.KVPool(e, dc, 128)
        s = abi.Sampler(e, 8, 4, CFG["vocab_size"])
        sch = abi.Scheduler(t, tpool, d, dpool, s, 4, 0.8, 77)
        if shard:
            sch.set_draft_shard(e, rank, WORLD)
        rng = np.random.default_rng(5)
        for i in range(5):  # different lengths and budgets: slices move as sequences finish
            sch.submit(rng.integers(0, CFG["vocab_size"], 10 + 7 * i).tolist(), max_tokens=12 + 5 * i,
                       stop_token=-1, seq_id=i)
        for _ in range(200):
            if sch.running() == 0 and sch.waiting() == 0:
                break
            sch.step()
        out = [sch.generated(i) for i in range(5)]
        err = e.device_error()
        sch.close()
        s.close()
        dpool.close()
        tpool.close()
        d.close()
        t.close()
        e.close()
        q.put((rank, out, err, None))
    except Exception as ex:
        q.put((rank, None, None, repr(ex)))


def test_tp2_sharded_drafting_tokens_equal_replicated():
    """Sequence-sharded drafting (each rank drafts and verifies its slice, drafts and
    results all-gathered) emits exactly the tokens of every rank drafting every
    sequence: the draft's fp32 results do not depend on the batch it runs in, and
    the uniforms are keyed by sequence id, not by rank."""
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    runs = {}
    for shard in (False, True):
        uid = abi.tp_unique_id()
        q = ctx.Queue()
        procs = [ctx.Process(target=_spec_worker, args=(r, uid, q, shard)) for r in range(WORLD)]
        for p in procs:
            p.start()
        res = {}
        try:
            for _ in range(WORLD):
                rank, out, err, exc = q.get(timeout=240)
                res[rank] = (out, err, exc)
        finally:
            for p in procs:
                p.join(timeout=30)
                if p.is_alive():
                    p.kill()
        for rank in range(WORLD):
            assert res[rank][2] is None, res[rank][2]
            assert res[rank][1] == 0
        assert res[0][0] == res[1][0]  # every rank holds the same tokens
        assert all(len(g) >= 12 for g in res[0][0])
        runs[shard] = res[0][0]
    assert runs[True] == runs[False]
