"""Benchmark: accepted tokens/s of the speculative draft->verify step.

Workload (the 8B/1B speculative configuration): Llama-3-8B-shape target
(32 layers, d 4096, 32/8 heads x 128, FFN 14336) with a Llama-3.2-1B-shape
draft (16 layers, d 2048, 32/8 x 64, FFN 8192), bf16 weights N(0, 0.02), fp32
accumulation, RoPE theta 5e5, vocab 128256, k = 5, temperature 0.8, 16-token
KV pages; 32 sequences per GPU with prompt lengths uniform in [512, 2048]
(random token ids), continuously batched.  Prefill is excluded: the prompts'
KV pages are allocated and filled with synthetic N(0, 1) values, then steady-
state speculative steps are timed.  A step = k draft forwards + k draft
samples + one (k+1)-token target verify forward + rejection sampling + cache
rollback, driven by libyk_host.so's Scheduler through the C-ABI.

Multi-GPU: one process per GPU (torchrun), each an independent replica with
its own 32 sequences (weak scaling, no data-path collective); the timed region
is bracketed by barriers and the max over ranks is reported.

--impl reference: the reference's CPU implementation of the same step (the
oracle restatement, all host threads), one bounded sample per step.

Other workloads (--workload): sampler (the rejection-sampling phase alone, 64
sequences, k=4, V=128256), gemma (Gemma-2-9B/2B shape, 64 sequences, split KV
pools), 70b-tp (70B-shape target tensor-parallel over all ranks, drafting
sharded by sequence), prefill (the first scheduler step of a fresh batch).
Under more than one GPU the 8b-dp run also times a global batch of 32 split
over the ranks (the line's `strong` object).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TARGET = dict(vocab_size=128256, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336,
              rope_theta=500000.0, rms_eps=1e-5, attn_cap=0.0, final_cap=0.0, window=0, window_layer_parity=-1,
              act=0, ref_compat=0)
DRAFT = dict(TARGET, d_model=2048, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64, ffn_dim=8192)
# --workload 70b-tp: Llama-3-70B-shape target, tensor parallel over all ranks, 8B-shape draft replicated
GEMM_TRAFFIC_RATIO = 1.018  # measured DRAM bytes / algorithmic bytes of a GEMM launch (ncu capture)
TARGET_70B = dict(TARGET, d_model=8192, n_layers=80, n_heads=64, n_kv_heads=8, head_dim=128, ffn_dim=28672)
METRIC_70B = "accepted tokens/sec, 70B-shape target (TP over all GPUs) + 8B-shape draft, k=4 batch 128"
WORKLOAD_70B = ("spec-decode step: 70B-shape target tensor-parallel (all-reduce over NVLink after o_proj / down_proj) + "
                "8B-shape draft replicated on every rank, each rank drafting its slice of the sequences, bf16, k=4, "
                "T=0.8, 128 seqs x 4096 ctx")
METRIC = "accepted tokens/sec, 8B/1B-shape k=5 batch 32, at 1/2/4/8 B200; verify HBM GB/s"
WORKLOAD = "spec-decode step: 8B-shape target + 1B-shape draft, bf16, k=5, T=0.8, 32 seqs/GPU, ctx U[512,2048]"
# --workload gemma: Gemma-2-9B-shape target with a Gemma-2-2B-shape draft
GEMMA_TARGET = dict(vocab_size=256000, d_model=3584, n_layers=42, n_heads=16, n_kv_heads=8, head_dim=256,
                    ffn_dim=14336, rope_theta=10000.0, rms_eps=1e-6, attn_cap=50.0, final_cap=30.0, window=4096,
                    window_layer_parity=0, act=1, ref_compat=0)
GEMMA_DRAFT = dict(GEMMA_TARGET, d_model=2304, n_layers=26, n_heads=8, n_kv_heads=4, ffn_dim=9216)
METRIC_GEMMA = "accepted tokens/sec, Gemma-2-9B/2B-shape k=4 batch 64, ctx U[2k,8k]"
WORKLOAD_GEMMA = ("spec-decode step: Gemma-2-9B-shape target + 2B-shape draft, bf16, GeGLU, attention cap 50, final "
                  "cap 30, window 4096 on even layers (split KV pools, out-of-window pages reclaimed), V=256000, k=4, "
                  "T=1.0, 64 seqs/GPU, ctx U[2048,8192]")
METRIC_STRONG = "accepted tokens/sec, 8B/1B-shape k=5, global batch 32 split across the GPUs"
METRIC_SAMPLER = "accepted tokens/sec, rejection sampling only: 64 seqs, k=4, V=128256, fp32 N(0,2^2) logits, T=1"
WORKLOAD_SAMPLER = ("sampler phase: draft sampling of k=4 tokens per sequence from fp32 draft logits + "
                    "verifySequence against fp32 target logits, 64 seqs/GPU, V=128256, T=1.0")
METRIC_PREFILL = "prompt tokens/sec, first scheduler step (whole prompts), 8B/1B-shape k=5 batch 32"
WORKLOAD_PREFILL = ("prefill step: the first Scheduler.step of 32 new sequences per GPU with U[512,2048]-token "
                    "prompts: both models over the whole prompts, then one draft / verify round; bf16, k=5, T=0.8")


def params_bytes(c: dict, es: int = 2) -> float:
    d, dh, F, V, L = c["d_model"], c["head_dim"], c["ffn_dim"], c["vocab_size"], c["n_layers"]
    per_layer = d * (c["n_heads"] + 2 * c["n_kv_heads"]) * dh + c["n_heads"] * dh * d + 3 * F * d
    return float(L * per_layer + V * d) * es  # streamed weights (LM head included; embedding is a gather)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = devices
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", ",".join(map(str, self.devices))],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (the reference's algorithm restated in C++), timed
# on a bounded sample of one step and extrapolated layer-by-layer.
# ---------------------------------------------------------------------------
def _tiled(rng, shape, std: float) -> np.ndarray:
    """An array of `shape` filled by repeating one 1 Mi-value N(0, std) block: the
    values do not change the oracle's CPU time, and drawing ~400 M normals per
    model would take longer than the timed work."""
    base = rng.standard_normal(1 << 20, dtype=np.float32) * np.float32(std)
    out = np.empty(int(np.prod(shape)), np.float32)
    full = out.size // base.size * base.size
    out[:full].reshape(-1, base.size)[:] = base
    out[full:] = base[: out.size - full]
    return out.reshape(shape)


def _oracle_layer_model(oracle, cfg: dict, n_layers: int, vocab: int, rng):
    c = dict(cfg, n_layers=n_layers, vocab_size=vocab)
    d, dh, F = c["d_model"], c["head_dim"], c["ffn_dim"]
    H, Hkv = c["n_heads"], c["n_kv_heads"]

    def nrm(*s):
        return _tiled(rng, s, 0.02)

    w = dict(embed=nrm(vocab, d), lm_head=nrm(vocab, d), final_norm=np.ones(d, np.float32))
    for name, shp in (("wq", (H * dh, d)), ("wk", (Hkv * dh, d)), ("wv", (Hkv * dh, d)), ("wo", (d, H * dh)),
                      ("wg", (F, d)), ("wu", (F, d)), ("wd", (d, F))):
        w[name] = [nrm(*shp) for _ in range(n_layers)]
    w["n1"] = [np.ones(d, np.float32) for _ in range(n_layers)]
    w["n2"] = [np.ones(d, np.float32) for _ in range(n_layers)]
    return c, w


_SAMPLE_MODELS: dict = {}
SAMPLE_FRACTION = 16  # one CPU sample = 1/16 of a step's work in every part


def cpu_step_sample(ctx_lens, k: int, T: float, nthreads: int, seed: int = 0) -> dict:
    """Times the oracle on 1/16 of one speculative step, every part cut by the
    same factor: 2 of the 32 target layers at the verify shape, 1/16 of the
    target LM head's vocabulary rows, for each of the k draft iterations 1 of the
    16 draft layers and 1/16 of the draft LM head, and the sampler phase of 2 of
    the 32 sequences.  Returns the timed seconds and, from an untimed sampler run
    over all the sequences, the tokens a whole step emits."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_ffi as oracle

    rng = np.random.default_rng(seed)
    B = len(ctx_lens)
    F = SAMPLE_FRACTION
    out = {}

    def time_forward(cfg, n_layers, vocab, n_new, last_n):
        blocks = [int(np.ceil((L + n_new) / 16)) for L in ctx_lens] if n_layers else [1] * B
        key = (tuple(sorted(cfg.items())), n_layers, vocab, n_new, tuple(blocks), nthreads)
        if key not in _SAMPLE_MODELS:  # built once per process: steps after the first time only the oracle
            c, w = _oracle_layer_model(oracle, cfg, n_layers, vocab, np.random.default_rng(1234))
            om = oracle.OracleModel(c, w, max(int(sum(blocks)), 1), nthreads=nthreads)
            if n_layers:
                om.pool[:] = _tiled(np.random.default_rng(4321), om.pool.size, 1.0)
            _SAMPLE_MODELS[key] = om
        om = _SAMPLE_MODELS[key]
        bt = np.zeros((B, max(blocks)), np.int32)
        nxt = 0
        for b, n in enumerate(blocks):
            bt[b, :n] = np.arange(nxt, nxt + n)
            nxt += n
        toks = rng.integers(0, vocab, B * n_new).tolist()
        qs = list(range(0, B * n_new + 1, n_new))
        ctx = [(L + n_new) if n_layers else n_new for L in ctx_lens]
        t0 = time.perf_counter()
        om.forward(toks, qs, ctx, bt, last_n=last_n)
        return time.perf_counter() - t0

    V = TARGET["vocab_size"]
    n_t = TARGET["n_layers"] // F
    out["target_layers_s"] = time_forward(TARGET, n_t, 2, k + 1, k + 1)
    out["target_lm_slice_s"] = time_forward(TARGET, 0, V // F, k + 1, k + 1)
    out["draft_s"] = 0.0
    for _ in range(k):
        out["draft_s"] += time_forward(DRAFT, DRAFT["n_layers"] // F, 2, 1, 1)
        out["draft_s"] += time_forward(DRAFT, 0, V // F, 1, 1)
    # sampler phase of B / F sequences on logits with the spread of random-init
    # models (std 0.02 * sqrt(d) ~ 1.3)
    bs = max(1, B // F)
    dl = rng.standard_normal((bs, k, V), dtype=np.float32) * np.float32(1.3)
    tl = rng.standard_normal((bs, k + 1, V), dtype=np.float32) * np.float32(1.3)
    t0 = time.perf_counter()
    _, _, cnt = oracle.spec_sample_batch(dl, tl, T, 1, seed, np.arange(bs, dtype=np.uint32), nthreads)
    out["sampler_s"] = time.perf_counter() - t0
    # the tokens a whole step emits, from the same sampler over all B sequences (untimed)
    dla = rng.standard_normal((B, k, V), dtype=np.float32) * np.float32(1.3)
    tla = rng.standard_normal((B, k + 1, V), dtype=np.float32) * np.float32(1.3)
    _, _, cnta = oracle.spec_sample_batch(dla, tla, T, 1, seed + 7919, np.arange(B, dtype=np.uint32), nthreads)
    out["sampled_seqs"] = B
    out["sampled_emitted"] = float(cnta.sum())
    out["sample_s"] = out["target_layers_s"] + out["target_lm_slice_s"] + out["draft_s"] + out["sampler_s"]
    return out


def cpu_sample_value(samples: list, B: int) -> tuple[float, float]:
    """(tokens/s of the timed samples, emitted tokens per full step): the step's
    emitted tokens are estimated from every sampled sequence; a sample carries
    1/16 of them, so its throughput is (emitted per step / 16) / sample time."""
    per_seq = sum(x["sampled_emitted"] for x in samples) / max(1, sum(x["sampled_seqs"] for x in samples))
    emitted = per_seq * B
    sample_s = float(np.mean([x["sample_s"] for x in samples]))
    return emitted / SAMPLE_FRACTION / sample_s, emitted


def cpu_baseline_dict(samples: list, nthreads: int, B: int) -> dict:
    val, emitted = cpu_sample_value(samples, B)
    ms = 1e3 * float(np.mean([x["sample_s"] for x in samples]))
    return {
        "value": val,
        "unit": "tokens/s",
        "cores": nthreads,
        "kind": "port",
        "sample": ("oracle (C++ restatement of S/SpeculativeSampler.swift, the draft sampling of "
                   "S/Scheduler.swift and the fp32 verify forward, all host threads) timed on 1/16 of a step in "
                   "every part: 2 of 32 target layers at the verify shape, 1/16 of the target LM head, per draft "
                   "iteration 1 of 16 draft layers and 1/16 of the draft LM head, the sampler phase of 2 of the "
                   f"32 sequences; {ms:.0f} ms per sample, throughput = (emitted tokens per step / 16) / sample "
                   f"time, {emitted:.1f} emitted tokens per step estimated by the oracle sampler over all "
                   f"32 sequences of every sample (untimed)"),
        "extrapolated_full_step_ms": ms * SAMPLE_FRACTION,
    }


# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allreduce_max(world, x: float) -> float:
    from yanaiengine_b200 import dp

    return dp.all_max(world, x)


def allreduce_sum(world, x: float) -> float:
    from yanaiengine_b200 import dp

    return dp.all_sum(world, x)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def run_yk(args, world, rank, local):
    """The speculative step: the weak-scaling headline (B sequences per GPU) and,
    on more than one GPU, the same job at a fixed global batch of `strong_batch`
    sequences split across the ranks (strong scaling); one engine and one pair of
    models per rank serve both."""
    from yanaiengine_b200 import abi, dp

    k, B, T = args.k, args.batch, args.temperature
    tp = args.workload == "70b-tp"
    eng = abi.Engine(local)
    if tp:
        # every rank holds one shard of the target and runs the whole batch
        import torch
        import torch.distributed as dist

        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(abi.tp_unique_id()), dtype=torch.uint8))
        if world > 1:
            dist.broadcast(uid, 0)
        eng.tp_init(bytes(uid.cpu().numpy()), rank, world)
        tcfg = abi.make_config(**TARGET_70B, dtype=abi.DTYPE_BF16, max_tokens=B * (k + 1) + 64, max_seqs=B)
        dcfg = abi.make_config(**TARGET, dtype=abi.DTYPE_BF16, max_tokens=B * 2 + 64, max_seqs=B)
    else:
        gem = args.workload == "gemma"
        tcfg = abi.make_config(**(GEMMA_TARGET if gem else TARGET), dtype=abi.DTYPE_BF16, max_tokens=B * (k + 1) + 64,
                               max_seqs=B)
        dcfg = abi.make_config(**(GEMMA_DRAFT if gem else DRAFT), dtype=abi.DTYPE_BF16, max_tokens=B * 2 + 64,
                               max_seqs=B)
    target = abi.Model(eng, tcfg, seed=1, init_std=0.02, tp=(rank, world) if tp else None)
    draft = abi.Model(eng, dcfg, seed=2, init_std=0.02)
    try:
        if tp:
            lens, mine = np.full(B, 4096, dtype=np.int64), np.arange(B)
            res = spec_phase(args, world, rank, local, eng, target, draft, lens, mine, B,
                             np.random.default_rng(7), profile=True)
        else:
            # the job's B x world sequences, split across ranks longest-first (B per rank)
            glens = (dp.global_lengths(B, world, seed=7, lo=2048, hi=8192) if args.workload == "gemma"
                     else dp.global_lengths(B, world, seed=7))
            mine = dp.partition(glens, world)[rank]
            lens = glens[mine]
            res = spec_phase(args, world, rank, local, eng, target, draft, lens, mine, B,
                             np.random.default_rng(7 + 1000 * rank), profile=True)
            if res is not None:
                res["config"]["global_batch"] = B * world
            if world > 1 and args.strong_batch > 0 and args.workload == "8b-dp":
                # strong scaling: the fixed global batch, strong_batch / world sequences per rank
                G = args.strong_batch
                sg = dp.global_lengths(-(-G // world), world, seed=7)[:G]
                smine = dp.partition(sg, world)[rank]
                st = spec_phase(args, world, rank, local, eng, target, draft, sg[smine], smine, len(smine),
                                np.random.default_rng(9 + 1000 * rank), profile=False)
                if rank == 0:
                    res["strong"] = {k2: st[k2] for k2 in ("value", "ms_per_step", "e2e", "gpu_launches",
                                                          "emitted_per_step", "verify_step", "accept_rate")}
                    res["strong"].update({"scaling": "strong", "global_batch": G,
                                          "seqs_per_gpu": f"{G // world}-{-(-G // world)}",
                                          "unit": "tokens/s", "metric": METRIC_STRONG})
    finally:
        draft.close()
        target.close()
        eng.close()
    return res, lens


def spec_phase(args, world, rank, local, eng, target, draft, lens, mine, B, rng, profile: bool):
    """Warm-up and K timed steps of one batch (its own KV pools, sampler and
    scheduler, freed at the end); with `profile`, also the per-launch roofline
    pass.  Returns the bench line (rank 0) or None."""
    from yanaiengine_b200 import abi

    import torch

    k, T = args.k, args.temperature
    tp = args.workload == "70b-tp"
    split = args.workload == "gemma"  # alternating windows: split pools, out-of-window pages reclaimed
    V = target.cfg.vocab_size
    grow = (args.warmup + 2 * args.steps + 4) * (k + 1) + 32
    blocks = int(sum(np.ceil((lens + grow) / 16))) + 64
    shard = tp and world > 1 and not args.no_draft_shard  # each rank drafts its slice of the batch
    # with sharded drafting the draft pool holds one slice (the longest sequences, to be safe)
    dblocks = (int(sum(np.sort(np.ceil((lens + grow) / 16))[::-1][: -(-len(lens) // world)])) + 64 if shard
               else blocks)
    twpool = dwpool = None
    if split:
        wblocks = len(lens) * (int(np.ceil((target.cfg.window + 2 * (k + 1) + 32) / 16)) + 2) + 64
        tpool = abi.KVPool(eng, target.cfg, blocks, abi.POOL_GLOBAL_LAYERS)
        twpool = abi.KVPool(eng, target.cfg, wblocks, abi.POOL_WINDOWED_LAYERS)
        dpool = abi.KVPool(eng, draft.cfg, blocks, abi.POOL_GLOBAL_LAYERS)
        dwpool = abi.KVPool(eng, draft.cfg, wblocks, abi.POOL_WINDOWED_LAYERS)
    else:
        tpool = abi.KVPool(eng, target.cfg, blocks)
        dpool = abi.KVPool(eng, draft.cfg, dblocks)
    sampler = abi.Sampler(eng, B, k, V)
    sch = None
    try:
        tpool.fill_random(11 + (rank if tp else 0), 1.0)
        dpool.fill_random(12, 1.0)
        if split:
            twpool.fill_random(13, 1.0)
            dwpool.fill_random(14, 1.0)
        sch = abi.Scheduler(target, tpool, draft, dpool, sampler, k, T, 1234 + (0 if tp else rank),
                            twpool=twpool, dwpool=dwpool)
        if shard:
            sch.set_draft_shard(eng, rank, world)
        for i, L in enumerate(lens):
            sch.submit(rng.integers(0, V, int(L)).tolist(), max_tokens=1 << 30, stop_token=-1,
                       seq_id=int(mine[i]), cached=True)
        for _ in range(args.warmup):
            sch.step()
        eng.sync()

        torch.cuda.set_device(local)
        stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks = ClockSampler(list(range(world)) if rank == 0 else [local])
        if rank == 0:
            clocks.start()
            time.sleep(0.5)
        _, em0, acc0 = sch.counters()
        launches0 = eng.launches()
        h2d = d2h = 0
        barrier(world)
        eng.sync()
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(args.steps):
            n_running = sch.running()
            # per-step host traffic through the C-ABI: token ids, positions, page tables in; tokens out
            sch.step()
            h2d += n_running * (2 * (k + 1) + 8) * 4 * (k + 1)
            d2h += n_running * (k + 2) * 4 * (k + 1)
        ev1.record(stream)
        eng.sync()
        wall = time.perf_counter() - t0
        barrier(world)
        dev_ms = ev0.elapsed_time(ev1)
        clk = clocks.stop() if rank == 0 else None
        _, em1, acc1 = sch.counters()
        emitted = em1 - em0
        launches = eng.launches() - launches0
        max_dev_s = allreduce_max(world, dev_ms / 1e3)
        max_wall = allreduce_max(world, wall)
        # data parallel: every rank emits its own sequences' tokens; tensor parallel:
        # all ranks emit the same tokens, counted once
        tot_emitted = float(emitted) if tp else allreduce_sum(world, float(emitted))
        tot_accepted = float(acc1 - acc0) if tp else allreduce_sum(world, float(acc1 - acc0))
        tot_seqs = float(B) if tp else allreduce_sum(world, float(B))

        gemm = attn = ar = None
        prof_steps = max(1, min(args.steps, 4))
        if profile:
            # kernel roofline: a second pass of the same steps with per-launch CUDA events
            eng.profile(True)
            for _ in range(prof_steps):
                sch.step()
            gemm = eng.profile_read(0)
            attn = eng.profile_read(1)
            ar = eng.profile_read(3)  # tensor-parallel all-reduce (own kernel or NCCL), if any
            eng.profile(False)
        # in-situ breakdown of one more step from the launch trace (first CTA past the
        # grid dependency wait, last CTA exit per launch), programmatic launch on
        ctx_before = [int(L) + len(sch.generated(int(sid))) for L, sid in zip(lens, mine)]
        breakdown = trace_breakdown(eng, sch)
    finally:
        if sch is not None:
            sch.close()
        sampler.close()
        for p in (dwpool, twpool, dpool, tpool):
            if p is not None:
                p.close()

    peaks = measured_peaks()
    if rank != 0:
        return None
    step_ms = max_dev_s * 1e3 / args.steps
    tcfg_d = TARGET_70B if tp else GEMMA_TARGET if split else TARGET
    res = {
        "metric": METRIC_70B if tp else METRIC_GEMMA if split else METRIC,
        "value": tot_emitted / max_dev_s,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "strong" if tp else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: random-init weights N(0,0.02), random token ids, synthetic N(0,1) KV context",
        "config": ({"workload": WORKLOAD_70B if not args.no_draft_shard else
                    WORKLOAD_70B.replace("each rank drafting its slice of the sequences", "every rank drafting every "
                                         "sequence"),
                    "global_batch": B, "k": k, "temperature": T, "ctx": "4096 + growth",
                    "parallelism": f"tp{world} target, draft replicated, drafting "
                                   f"{'of every sequence on every rank' if args.no_draft_shard else 'sharded by sequence'}",
                    "l2": "inputs larger than L2 (17.5 GB target shard + 16 GB draft per GPU per step)"}
                   if tp else
                   {"workload": WORKLOAD_GEMMA if split else WORKLOAD, "global_batch": B * world, "seqs_per_gpu": B,
                    "k": k, "temperature": T, "ctx": ("U[2048,8192]" if split else "U[512,2048]") + " + growth",
                    "parallelism": f"dp{world} (replicas)",
                    "l2": "inputs larger than L2 (GBs of weights streamed per step)"}),
        "e2e": {"value": tot_emitted / max_wall, "unit": "tokens/s", "h2d_bytes_per_step": int(h2d / args.steps),
                "d2h_bytes_per_step": int(d2h / args.steps)},
        "gpu_launches": int(launches),
        "accept_rate": float(tot_accepted / max(1.0, args.steps * tot_seqs * k)),
        "emitted_per_step": float(tot_emitted / args.steps),
        "verify_step": verify_roofline(tcfg_d, ctx_before, k, world if tp else 1,
                                       breakdown.get("verify_forward_us"), peaks),
        "step_breakdown": breakdown,
        "clocks": clk,
    }
    if gemm is not None:
        gemm_gbs = gemm["bytes"] / (gemm["ms"] / 1e3) / 1e9 if gemm["ms"] > 0 else 0.0
        attn_gbs = attn["bytes"] / (attn["ms"] / 1e3) / 1e9 if attn["ms"] > 0 else 0.0
        res["roofline"] = {"bound": "hbm", "achieved": gemm_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                           "frac": gemm_gbs / peaks["hbm_gbs"],
                           # ncu, 28672x4096x192 gate/up launch: DRAM read+write / algorithmic bytes = 1.018
                           "traffic": GEMM_TRAFFIC_RATIO * gemm["bytes"] / max(1, gemm["launches"]),
                           "traffic_src": "ncu dram bytes of the 28672x4096x192 gate/up launch / its algorithmic "
                                          "bytes (1.018), applied to the average launch's algorithmic bytes",
                           "kernel": "gemm_tc_kernel",
                           "peak_src": peaks["src"],
                           "launches": gemm["launches"],
                           "avg_launch_us": 1e3 * gemm["ms"] / max(1, gemm["launches"])}
        res["attention"] = {"achieved_gbs": attn_gbs, "frac": attn_gbs / peaks["hbm_gbs"],
                            "launches": attn["launches"]}
        if tp and ar is not None and ar["launches"] > 0:
            ar_ms = ar["ms"] / prof_steps
            res["allreduce"] = {
                "ms_per_step": ar_ms, "launches_per_step": ar["launches"] / prof_steps,
                "share_of_step": ar_ms / step_ms,
                "payload": "fp32" if os.environ.get("YK_TP_PAYLOAD") == "f32" else "bf16",
                "kind": ("ncclAllReduce" if os.environ.get("YK_TP_AR") == "nccl" or os.environ.get("YK_TP_PAYLOAD") == "f32"
                         else "own kernel over NVLink peer memory, "
                         + ("one shot" if world == 2 and os.environ.get("YK_TP_AR") != "twoshot" else "two-shot")),
                # what one rank sends over NVLink in a ring all-reduce, per second of all-reduce time
                "link_gbs": ar["bytes"] / (ar["ms"] / 1e3) / 1e9 if ar["ms"] > 0 else None,
                "link_peak_gbs": 770.0,
                "note": "CUDA events around each all-reduce on the engine stream, in a second pass of "
                        f"{prof_steps} steps without programmatic launch"}
    return res


def verify_roofline(cfg: dict, ctx_before, k: int, tp_world: int, us, peaks) -> dict | None:
    """HBM roofline of the verify forward (the target's pass over the k + 1 new
    tokens of every sequence), timed in situ from the launch trace: algorithmic
    bytes = the target's streamed weights (LM head included; this rank's shard
    under tensor parallelism) + every sequence's KV context read once (the new
    tokens' K/V included)."""
    if not us:
        return None
    kv_layer_tok = 2 * cfg["n_kv_heads"] // tp_world * cfg["head_dim"] * 2  # bytes per token per layer (K and V)
    w = params_bytes(cfg) - cfg["vocab_size"] * cfg["d_model"] * 2  # sharded part
    weights = w / tp_world + cfg["vocab_size"] * cfg["d_model"] * 2
    L, W, par = cfg["n_layers"], cfg.get("window", 0), cfg.get("window_layer_parity", -1)
    n_win = 0 if W <= 0 else (L if par < 0 else sum(1 for l in range(L) if l % 2 == par))
    # a windowed layer reads the keys inside the window of its queries (the last
    # query's window plus the k earlier new tokens)
    kv = sum((L - n_win) * (c + k + 1) + n_win * min(c + k + 1, W + k) for c in ctx_before) * kv_layer_tok
    ach = (weights + kv) / (us * 1e-6) / 1e9
    return {"us": us, "bytes": weights + kv, "weight_bytes": weights, "kv_bytes": kv, "achieved_gbs": ach,
            "peak_gbs": peaks["hbm_gbs"], "frac": ach / peaks["hbm_gbs"], "peak_src": peaks["src"]}


def run_sampler(args, world, rank, local):
    """--workload sampler: the rejection-sampling phase alone (draft sampling of
    k tokens per sequence from fp32 draft logits, then verifySequence against fp32
    target logits), 64 sequences per GPU, k = 4, V = 128256, logits i.i.d.
    N(0, 2^2), T = 1.  `value`: the logits stay resident on the device
    (yk_spec_sample_logits with NULL logits samples them again each step with a
    new step index, so new uniforms); `e2e`: every step uploads both logit
    tensors from pinned host memory through the same call."""
    from yanaiengine_b200 import abi

    import torch

    k, B, T = args.k, args.batch, args.temperature
    V = TARGET["vocab_size"]
    eng = abi.Engine(local)
    s = abi.Sampler(eng, B, k, V)
    try:
        rng = np.random.default_rng(1234 + rank)
        dl = torch.empty((B, k, V), dtype=torch.float32, pin_memory=True).numpy()
        tl = torch.empty((B, k + 1, V), dtype=torch.float32, pin_memory=True).numpy()
        dl[:] = rng.standard_normal((B, k, V), dtype=np.float32) * np.float32(2.0)
        tl[:] = rng.standard_normal((B, k + 1, V), dtype=np.float32) * np.float32(2.0)
        ids = np.arange(B, dtype=np.uint32) + np.uint32(B * rank)
        step_bytes = float(dl.nbytes + tl.nbytes)
        for w in range(args.warmup):
            s.sample_logits(dl, tl, T, 1234, 100000 + w, ids)
        torch.cuda.set_device(local)
        stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
        clocks = ClockSampler(list(range(world)) if rank == 0 else [local])
        if rank == 0:
            clocks.start()
            time.sleep(0.5)
        launches0 = eng.launches()
        # device-resident inputs
        barrier(world)
        eng.sync()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        emitted = 0
        ev0.record(stream)
        for i in range(args.steps):
            _, _, cnt = s.sample_logits(None, None, T, 1234, i, ids)
            emitted += int(cnt.sum())
        ev1.record(stream)
        eng.sync()
        dev_s = ev0.elapsed_time(ev1) / 1e3
        launches = eng.launches() - launches0
        # end to end: host logits uploaded inside every step
        barrier(world)
        t0 = time.perf_counter()
        em_e2e = 0
        for i in range(args.steps):
            _, _, cnt = s.sample_logits(dl, tl, T, 1234, args.steps + i, ids)
            em_e2e += int(cnt.sum())
        wall = time.perf_counter() - t0
        barrier(world)
        clk = clocks.stop() if rank == 0 else None
        # per-kernel shares of one more device-resident step (launch trace)
        n0 = eng.launches()
        eng.trace(64)
        s.sample_logits(None, None, T, 1234, 2 * args.steps, ids)
        rec, n1 = eng.trace_read()
        eng.trace(0)
        kinds = {}
        for i in range(n0, n1):
            r = rec[i % 64].astype(np.int64)
            name = TRACE_KINDS.get(int(r[3]) & 15, "other")
            kinds[name] = kinds.get(name, 0.0) + (r[2] - r[1]) / 1e3
        max_dev = allreduce_max(world, dev_s)
        max_wall = allreduce_max(world, wall)
        tot = allreduce_sum(world, float(emitted))
        tot_e2e = allreduce_sum(world, float(em_e2e))
    finally:
        s.close()
        eng.close()
    if rank != 0:
        return None, None
    peaks = measured_peaks()
    ms = max_dev * 1e3 / args.steps
    gbs = step_bytes / (ms / 1e3) / 1e9
    res = {
        "metric": METRIC_SAMPLER, "value": tot / max_dev, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: fp32 logits i.i.d. N(0, 2^2) (numpy seed 1234 + rank), Philox uniforms",
        "config": {"workload": WORKLOAD_SAMPLER, "global_batch": B * world, "seqs_per_gpu": B, "k": k, "vocab": V,
                   "temperature": T, "l2": "inputs larger than L2 (295 MB of logits per step)"},
        "e2e": {"value": tot_e2e / max_wall, "unit": "tokens/s", "h2d_bytes_per_step": int(step_bytes + 4 * B),
                "d2h_bytes_per_step": int(4 * (B * k + B * (k + 1) + B))},
        "gpu_launches": int(launches),
        "emitted_per_step": tot / args.steps,
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": None,
                     "kernel": "sampler phase: draft_partial_kernel, draft_prob_kernel, draft_sample_kernel, "
                               "verify_kernel (algorithmic bytes = both logit tensors read once per step)",
                     "peak_src": peaks["src"], "step_bytes": step_bytes},
        "kernel_us": {k2: round(v, 1) for k2, v in kinds.items()},
        "clocks": clk,
    }
    return res, None


def sampler_cpu_baselines(args) -> dict:
    """The oracle sampler (draft sampling + verifySequence, the reference's
    SpeculativeSampler restated) on one step of the same workload: one thread
    (the reference loops over sequences serially) and every host thread."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_ffi as oracle

    k, B, T, V = args.k, args.batch, args.temperature, TARGET["vocab_size"]
    rng = np.random.default_rng(1234)
    dl = rng.standard_normal((B, k, V), dtype=np.float32) * np.float32(2.0)
    tl = rng.standard_normal((B, k + 1, V), dtype=np.float32) * np.float32(2.0)
    ids = np.arange(B, dtype=np.uint32)
    out = {}
    for nt in (1, os.cpu_count() or 1):
        t0 = time.perf_counter()
        _, _, cnt = oracle.spec_sample_batch(dl, tl, T, 1234, 0, ids, nt)
        dt = time.perf_counter() - t0
        out[nt] = {"value": float(cnt.sum()) / dt, "unit": "tokens/s", "cores": nt, "kind": "port",
                   "sample": f"oracle sampler phase on one step of {B} sequences (k={k}, V={V}): {dt * 1e3:.0f} ms"}
    return out


def reference_sampler(args, world, nthreads):
    """--impl reference --workload sampler: the oracle sampler (the reference's
    SpeculativeSampler restated) on the same workload, all host threads, one
    whole step per timed step."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_ffi as oracle

    k, B, T, V = args.k, args.batch, args.temperature, TARGET["vocab_size"]
    rng = np.random.default_rng(1234)
    dl = rng.standard_normal((B, k, V), dtype=np.float32) * np.float32(2.0)
    tl = rng.standard_normal((B, k + 1, V), dtype=np.float32) * np.float32(2.0)
    ids = np.arange(B, dtype=np.uint32)
    for w in range(args.warmup):
        oracle.spec_sample_batch(dl, tl, T, 1234, 100000 + w, ids, nthreads)
    em, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        _, _, cnt = oracle.spec_sample_batch(dl, tl, T, 1234, i, ids, nthreads)
        em += int(cnt.sum())
    dt = time.perf_counter() - t0
    val = em / dt
    print(json.dumps({
        "metric": METRIC_SAMPLER, "value": val, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD_SAMPLER, "global_batch": B, "k": k, "vocab": V, "temperature": T},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                         "sample": f"oracle sampler phase, {args.steps} whole steps of {B} sequences"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def run_prefill(args, world, rank, local):
    """--workload prefill: the first scheduler step of a fresh batch (the reference
    feeds whole prompts there: S/Scheduler.swift:68-69,201-202).  Each timed step
    is a new scheduler over the same 32 prompt lengths per GPU (weak scaling);
    the KV pools and models are reused."""
    from yanaiengine_b200 import abi, dp

    import torch

    k, B, T = args.k, args.batch, args.temperature
    glens = dp.global_lengths(B, world, seed=7)
    mine = dp.partition(glens, world)[rank]
    lens = glens[mine]
    tot = int(lens.sum())
    eng = abi.Engine(local)
    tcfg = abi.make_config(**TARGET, dtype=abi.DTYPE_BF16, max_tokens=tot + B * (k + 1) + 64, max_seqs=B)
    dcfg = abi.make_config(**DRAFT, dtype=abi.DTYPE_BF16, max_tokens=tot + B * (k + 1) + 64, max_seqs=B)
    blocks = int(sum(np.ceil((lens + 2 * (k + 1) + 32) / 16))) + 64
    target = abi.Model(eng, tcfg, seed=1, init_std=0.02)
    draft = abi.Model(eng, dcfg, seed=2, init_std=0.02)
    tpool = abi.KVPool(eng, target.cfg, blocks)
    dpool = abi.KVPool(eng, dcfg, blocks)
    sampler = abi.Sampler(eng, B, k, TARGET["vocab_size"])
    rng = np.random.default_rng(7 + 1000 * rank)
    prompts = [rng.integers(0, TARGET["vocab_size"], int(L)).tolist() for L in lens]

    def fresh():
        sch = abi.Scheduler(target, tpool, draft, dpool, sampler, k, T, 1234 + rank)
        for i, pr in enumerate(prompts):
            sch.submit(pr, max_tokens=1 << 30, stop_token=-1, seq_id=int(mine[i]))
        return sch

    for _ in range(args.warmup):
        sch = fresh()
        sch.step()
        sch.close()
    eng.sync()
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
    clocks = ClockSampler(list(range(world)) if rank == 0 else [local])
    if rank == 0:
        clocks.start()
        time.sleep(0.5)
    launches0 = eng.launches()
    dev_ms = wall = 0.0
    h2d = 0
    barrier(world)
    for _ in range(args.steps):
        sch = fresh()
        eng.sync()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        ev0.record(stream)
        sch.step()
        ev1.record(stream)
        eng.sync()
        wall += time.perf_counter() - t0
        dev_ms += ev0.elapsed_time(ev1)
        # prompts (target and draft), positions and page tables in; tokens out
        h2d += 2 * (tot + B * (k + 1)) * 4 * 3
        sch.close()
    barrier(world)
    clk = clocks.stop() if rank == 0 else None
    launches = eng.launches() - launches0
    max_dev_s = allreduce_max(world, dev_ms / 1e3)
    max_wall = allreduce_max(world, wall)
    tot_tokens = allreduce_sum(world, float(tot * args.steps))
    # tensor roofline of the GEMMs: one more step with per-launch CUDA events
    eng.profile(True)
    sch = fresh()
    sch.step()
    sch.close()
    gemm = eng.profile_read(0)
    attn = eng.profile_read(1)
    eng.profile(False)
    peaks = measured_peaks()
    res = None
    if rank == 0:
        tflops = gemm["flops"] / (gemm["ms"] / 1e3) / 1e12 if gemm["ms"] > 0 else 0.0
        res = {
            "metric": METRIC_PREFILL, "value": tot_tokens / max_dev_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_dev_s * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init weights N(0,0.02), random prompt token ids",
            "config": {"workload": WORKLOAD_PREFILL, "global_batch": B * world, "seqs_per_gpu": B,
                       "prompt_tokens_per_gpu": tot, "k": k, "temperature": T, "parallelism": f"dp{world} (replicas)",
                       "l2": "inputs larger than L2 (weights and prompts stream once per step)"},
            "e2e": {"value": tot_tokens / max_wall, "unit": "tokens/s", "h2d_bytes_per_step": int(h2d / args.steps),
                    "d2h_bytes_per_step": int(B * (k + 2) * 4 * (k + 1))},
            "gpu_launches": int(launches),
            # the GEMMs run back to back inside a ~1 s step under the power cap: the
            # sustained cuBLAS figure is the denominator (the burst one beside it)
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops_sustained"],
                         "unit": "TFLOP/s", "frac": tflops / peaks["bf16_tflops_sustained"],
                         "frac_of_burst": tflops / peaks["bf16_tflops"], "traffic": None, "kernel": "gemm_tc_kernel",
                         "peak_src": peaks["src"] + " (sustained: a seconds-long step under the power cap)",
                         "share_of_step": gemm["ms"] / (max_dev_s * 1e3 / args.steps),
                         "launches": gemm["launches"], "avg_launch_us": 1e3 * gemm["ms"] / max(1, gemm["launches"])},
            "attention": {"ms": attn["ms"], "launches": attn["launches"]},
            "cpu_baseline": None,
            "clocks": clk,
        }
    sampler.close()
    dpool.close()
    tpool.close()
    draft.close()
    target.close()
    eng.close()
    return res, lens


TRACE_KINDS = {1: "embed", 2: "rmsnorm", 3: "gemm", 4: "attention", 5: "draft_sample", 6: "row_stats", 7: "verify"}


EPI_NAMES = {0: "store", 1: "qkv", 2: "resid", 3: "glu", 4: "logits"}


def trace_name(k: int) -> str:
    base = TRACE_KINDS.get(k & 15, "other")
    if base == "gemm":
        name = f"gemm_{EPI_NAMES.get((k >> 4) & 15, '?')}_{128 * ((k >> 8) & 0xFFFF)}x{16 * ((k >> 24) & 0x7F)}"
        return name + "+down" if k >> 31 else name  # bit 31: the chained gate/up + down_proj launch
    if base == "attention":
        return f"attention_dh{k >> 8}"
    return base


def trace_breakdown(eng, sch, cap: int = 8192) -> dict:
    """One step under the launch trace.  Each launch's share of the step is
    end[i] - end[i-1] (its kernels finish in stream order), attributed to its kind;
    `idle` is the part of that share before its first CTA got past the dependency
    wait (launch latency, host work between forward calls)."""
    n0 = eng.launches()
    eng.trace(cap)
    sch.step()
    rec, n1 = eng.trace_read()
    eng.trace(0)
    ids = [i % cap for i in range(n0, n1)]
    if not ids or n1 - n0 > cap:
        return {}
    r = rec[ids].astype(np.int64)
    start, end, kind = r[:, 1], r[:, 2], r[:, 3]
    span = float(end.max() - start[0])
    out = {"step_us": span / 1e3, "launches": int(len(ids)), "busy_us": {}, "idle_us": 0.0, "count": {}}
    prev_end = start[0]
    names, shares = [], []
    for k, s0, e0 in zip(kind, start, end):
        share = max(0, e0 - prev_end)
        idle = min(share, max(0, s0 - prev_end))
        name = trace_name(int(k))
        names.append(name)
        shares.append(share)
        out["busy_us"][name] = out["busy_us"].get(name, 0.0) + (share - idle) / 1e3
        out["count"][name] = out["count"].get(name, 0) + 1
        out["idle_us"] += idle / 1e3
        prev_end = max(prev_end, e0)
    # the verify forward: the last embedding launch through the last LM-head GEMM (the
    # target's layers, its final norm and its logits; hand-offs included)
    last_lm = max((i for i, n in enumerate(names) if n.startswith("gemm_logits")), default=-1)
    first = max((i for i, n in enumerate(names[: last_lm + 1]) if n == "embed"), default=-1)
    if last_lm >= 0 and first >= 0:
        out["verify_forward_us"] = round(sum(shares[first: last_lm + 1]) / 1e3, 1)
    out["busy_us"] = {k: round(v, 1) for k, v in sorted(out["busy_us"].items(), key=lambda x: -x[1])}
    out["idle_us"] = round(out["idle_us"], 1)
    out["step_us"] = round(out["step_us"], 1)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="yk", choices=["yk", "reference"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--temperature", type=float, default=0.8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-draft-shard", action="store_true",
                    help="70b-tp: every rank drafts every sequence (default: each rank drafts its slice)")
    ap.add_argument("--strong-batch", type=int, default=32,
                    help="8b-dp on more than one GPU: also time this global batch split across the GPUs "
                         "(strong scaling, reported as `strong`); 0 skips it")
    ap.add_argument("--workload", default="8b-dp", choices=["8b-dp", "70b-tp", "prefill", "sampler", "gemma"],
                    help="8b-dp: the headline 8B/1B data-parallel step; 70b-tp: 70B-shape target over all GPUs; "
                         "prefill: the first scheduler step of a fresh batch (whole prompts); sampler: the "
                         "rejection-sampling phase alone (64 seqs, k=4, V=128256, fp32 N(0,4) logits); gemma: "
                         "the Gemma-2-9B/2B-shape step (64 seqs/GPU, k=4, T=1, ctx U[2k,8k], split KV pools)")
    args = ap.parse_args()
    if args.workload == "sampler":
        # the sampler-only configuration: 64 sequences, k = 4, T = 1 (other flags as given)
        if "--batch" not in sys.argv:
            args.batch = 64
        if "--k" not in sys.argv:
            args.k = 4
        if "--temperature" not in sys.argv:
            args.temperature = 1.0
    if args.workload == "gemma":
        # the Gemma configuration: 64 sequences, k = 4, T = 1 (other flags as given)
        if "--batch" not in sys.argv:
            args.batch = 64
        if "--k" not in sys.argv:
            args.k = 4
        if "--temperature" not in sys.argv:
            args.temperature = 1.0
    if args.workload == "70b-tp":
        # the 70B configuration: batch 128, k = 4 (other flags as given)
        if "--batch" not in sys.argv:
            args.batch = 128
        if "--k" not in sys.argv:
            args.k = 4
    nthreads = os.cpu_count() or 1

    if args.impl == "reference":
        # CPU only: no process group and no GPU; under torchrun rank 0 alone runs
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        if args.workload == "sampler":
            reference_sampler(args, world, nthreads)
            return
        lens = np.random.default_rng(7).integers(512, 2049, args.batch)
        for w in range(args.warmup):  # untimed: builds the sample models, primes caches and threads
            cpu_step_sample(lens, args.k, args.temperature, nthreads, seed=1000 + w)
        samples = [cpu_step_sample(lens, args.k, args.temperature, nthreads, seed=s) for s in range(args.steps)]
        cb = cpu_baseline_dict(samples, nthreads, args.batch)
        val = cb["value"]
        ms = 1e3 * float(np.mean([x["sample_s"] for x in samples]))
        print(json.dumps({
            "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": args.batch, "k": args.k,
                       "temperature": args.temperature,
                       "step": "each timed step is one 1/16-of-a-step sample (see cpu_baseline.sample)"},
            "extrapolated": True,
            "extrapolated_full_step_ms": ms * SAMPLE_FRACTION,
            "cpu_baseline": cb,
            "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    world, rank, local = dist_setup(args.gpus)
    run = {"prefill": run_prefill, "sampler": run_sampler}.get(args.workload, run_yk)
    res, lens = run(args, world, rank, local)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline and args.workload == "8b-dp":
            samples = [cpu_step_sample(lens, args.k, args.temperature, nthreads, seed=s) for s in range(2)]
            res["cpu_baseline"] = cpu_baseline_dict(samples, nthreads, args.batch)
        if world == 1 and not args.no_cpu_baseline and args.workload == "sampler":
            cb = sampler_cpu_baselines(args)
            res["cpu_baseline"] = cb[max(cb)]
            res["cpu_baseline_1thread"] = cb[1]
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
