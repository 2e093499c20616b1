"""Small single-kernel workloads for profiling (ncu) and timing.

    python -m yanaiengine_b200.kernel_cases attention [--dh 128 --group 4 --kv-heads 8 --seqs 32 --new 6]
    python -m yanaiengine_b200.kernel_cases gemm [--n 28672 --k 4096 --m 192]
    python -m yanaiengine_b200.kernel_cases sampler [--seqs 32 --k 5 --vocab 128256]
    python -m yanaiengine_b200.kernel_cases forward [--shape draft|target --layers 4 --steps 3]
    torchrun --nproc-per-node N -m yanaiengine_b200.kernel_cases allreduce [--tokens 16 80 128 640 --d 8192]

`attention` builds a 2-layer bf16 model whose attention has the verify shape of
the 8B-class target (or the 1B-class draft with --dh 64 --new 1, the Gemma-2 9B
target with --dh 256 --group 2 --seqs 64 --new 5 --ctx-lo 2048 --ctx-hi 8192),
fills a KV pool with a synthetic context of U[ctx-lo, ctx-hi] (default
U[512, 2048]) tokens per sequence and runs forward steps; the pool holds about 1 GB, one layer's KV (170 MB at the target
shape) is larger than L2.  `gemm` runs the tcgen05 GEMM test hook on one layer
shape with an L2 flush before each launch.  Both print one timing line.
`allreduce` times the tensor-parallel all-reduce of [tokens x d] bf16 alone,
the group's own kernel against ncclAllReduce.
"""
from __future__ import annotations

import argparse
import os
import time

import numpy as np

from . import abi


def attention(args) -> None:
    e = abi.Engine(0)
    H = args.kv_heads * args.group
    cfg = abi.make_config(vocab_size=1024, d_model=512, n_layers=2, n_heads=H, n_kv_heads=args.kv_heads,
                          head_dim=args.dh, ffn_dim=1024, rope_theta=500000.0, rms_eps=1e-5, dtype=abi.DTYPE_BF16,
                          max_tokens=max(64, args.seqs * args.new), max_seqs=args.seqs)
    rng = np.random.default_rng(0)
    ctx = rng.integers(args.ctx_lo, args.ctx_hi + 1, args.seqs)
    pages = [(int(c) + args.new * args.steps + 15) // 16 for c in ctx]
    nb = sum(pages) + 8
    m = abi.Model(e, cfg, seed=1)
    pool = abi.KVPool(e, cfg, nb)
    pool.fill_random(3, 1.0)
    tables = np.zeros((args.seqs, max(pages)), np.int32)
    nxt = 0
    for b, n in enumerate(pages):
        tables[b, :n] = np.arange(nxt, nxt + n)
        nxt += n
    if args.stamps:
        m.attention_stamps(4096)
    times = []
    for s in range(args.steps):
        toks = rng.integers(0, 1024, args.seqs * args.new).tolist()
        qs = list(range(0, args.seqs * args.new + 1, args.new))
        cl = (ctx + args.new * (s + 1)).tolist()
        e.sync()
        t0 = time.perf_counter()
        m.forward(pool, toks, qs, cl, tables, last_n=1)
        e.sync()
        times.append(time.perf_counter() - t0)
    kv = float(sum(ctx)) * 2 * args.kv_heads * args.dh * 2
    print(f"attention dh={args.dh} G={args.group} Hkv={args.kv_heads} seqs={args.seqs} new={args.new}: "
          f"{kv / 1e6:.0f} MB KV per layer, forward step {1e3 * min(times):.3f} ms (2 layers + GEMMs)")
    if args.stamps:
        st = m.attention_stamps().astype(np.int64)
        t0 = st[:, 0].min()
        start, first, loop, end = ((st[:, i] - t0) / 1e3 for i in range(4))
        pages = st[:, 4]
        end = np.where(st[:, 3] > 0, end, loop)
        print(f"  {len(st)} CTAs on {len(set(st[:, 5].tolist()))} SMs; kernel span {end.max():.1f} us")
        print(f"  start: median {np.median(start):.1f} max {start.max():.1f} us;"
              f" first page after start: median {np.median(first - start):.1f} us")
        busy = loop - first
        rate = pages * 16 * args.dh * 2 * 2 / np.maximum(busy, 1e-3) / 1e3  # K + V bytes per us -> GB/s
        print(f"  loop: median {np.median(busy):.1f} max {busy.max():.1f} us; per-CTA GB/s median {np.median(rate):.1f}"
              f" (pages median {np.median(pages):.0f} max {pages.max()}); merge+write median {np.median(end - loop):.1f} us")
        for q in (0.1, 0.5, 0.9, 1.0):
            print(f"  end quantile {q:.1f}: {np.quantile(end, q):.1f} us")
    pool.close()
    m.close()
    e.close()


def sampler(args) -> None:
    """Draft sampling of B x k rows and verification of B sequences from synthetic
    N(0, s^2) logits (s = --logit-std, default 2) (yk_spec_sample_logits), with per-CTA phase stamps."""
    e = abi.Engine(0)
    B, k, V = args.seqs, args.k, args.vocab
    rng = np.random.default_rng(0)
    dl = rng.normal(0, args.logit_std, (B, k, V)).astype(np.float32)
    tl = rng.normal(0, args.logit_std, (B, k + 1, V)).astype(np.float32)
    s = abi.Sampler(e, B, k, V)
    s.stamps(B * k)
    seq = np.arange(B, dtype=np.uint32)
    times = []
    for step in range(args.steps):
        t0 = time.perf_counter()
        s.sample_logits(dl, tl, args.temperature, 7, step, seq)
        times.append(time.perf_counter() - t0)
    d, v = s.stamps()
    d, v = d.astype(np.int64), v[:B].astype(np.int64)
    ph = lambda a, i, j: np.median((a[:, j] - a[:, i]) / 1e3)
    print(f"sampler B={B} k={k} V={V} T={args.temperature}: call {1e3 * min(times):.2f} ms (with host copies)")
    seq_d, ties_d = d[:, 6] & 0xFFFFFFFF, d[:, 6] >> 32
    ties_v = v[:, 6] >> 32
    print(f"  draft token CTAs {len(d)}: chain {ph(d, 2, 3):.1f} us "
          f"(max {np.max((d[:, 3] - d[:, 2]) / 1e3):.1f}); rounds median {np.median(d[:, 4]):.0f} max {d[:, 4].max()}, "
          f"special {np.median(d[:, 5]):.0f}, sequential {np.median(seq_d):.0f}, ties {np.median(ties_d):.0f}; "
          f"span {(d[:, 3].max() - d[:, 0].min()) / 1e3:.1f} us")
    print(f"  verify CTAs {len(v)}: total {ph(v, 0, 3):.1f} us (max {np.max((v[:, 3] - v[:, 0]) / 1e3):.1f}); "
          f"rounds median {np.median(v[:, 4]):.0f} max {v[:, 4].max()}, special {np.median(v[:, 5]):.0f}, "
          f"ties {np.median(ties_v):.0f}")
    s.close()
    e.close()


# Layer shapes of the speculative workload: the 1B-shape draft (decode, 1 new token
# per sequence) and the 8B-shape target (verify, k + 1 = 6 new tokens per sequence).
FWD_SHAPES = {
    "draft": (dict(vocab_size=128256, d_model=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn_dim=8192), 1),
    "target": (dict(vocab_size=128256, d_model=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336), 6),
}


def forward(args) -> None:
    """A few forwards of a `--layers`-layer model of the draft or target shape over
    32 sequences with U[512, 2048]-token synthetic contexts: every GEMM kind and the
    attention of that shape, in situ (the ncu target for one launch of a kind)."""
    e = abi.Engine(0)
    shape, new = FWD_SHAPES[args.shape]
    seqs = args.seqs
    cfg = abi.make_config(**shape, n_layers=args.layers, rope_theta=500000.0, rms_eps=1e-5, dtype=abi.DTYPE_BF16,
                          max_tokens=seqs * new + 64, max_seqs=seqs)
    m = abi.Model(e, cfg, seed=1, init_std=0.02)
    rng = np.random.default_rng(0)
    ctx = rng.integers(512, 2049, seqs)
    pages = [(int(c) + new * (args.steps + 1) + 15) // 16 for c in ctx]
    pool = abi.KVPool(e, cfg, sum(pages) + 8)
    pool.fill_random(3, 1.0)
    tables = np.zeros((seqs, max(pages)), np.int32)
    nxt = 0
    for b, n in enumerate(pages):
        tables[b, :n] = np.arange(nxt, nxt + n)
        nxt += n
    times = []
    for s in range(args.steps):
        toks = rng.integers(0, shape["vocab_size"], seqs * new).tolist()
        qs = list(range(0, seqs * new + 1, new))
        e.sync()
        t0 = time.perf_counter()
        m.forward(pool, toks, qs, (ctx + new * (s + 1)).tolist(), tables, last_n=1)
        e.sync()
        times.append(time.perf_counter() - t0)
    print(f"forward {args.shape} x {args.layers} layers, {seqs} seqs x {new} new tokens: "
          f"{1e3 * min(times):.3f} ms per forward")
    pool.close()
    m.close()
    e.close()


def gemm(args) -> None:
    e = abi.Engine(0)
    rng = np.random.default_rng(0)
    W = abi.bf16_bits(rng.normal(0, 0.05, (args.n, args.k)).astype(np.float32))
    X = abi.bf16_bits(rng.normal(0, 1, (args.m, args.k)).astype(np.float32))
    _, ms, _, g = abi.gemm_bf16_timed(e, W, X, 0, -args.reps)
    gb = (args.n + args.m) * args.k * 2 / 1e9
    print(f"gemm {args.n}x{args.k}x{args.m} grid={g}: {1e3 * ms:.1f} us cold-L2, {gb / (ms / 1e3):.0f} GB/s")
    e.close()


def allreduce(args) -> None:
    """The tensor-parallel all-reduce alone, under torchrun (one rank per GPU):
    per message size, the group's own kernel and ncclAllReduce, each timed over
    back-to-back calls (max over ranks)."""
    import datetime

    import torch
    import torch.distributed as dist

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        raise SystemExit("allreduce: run under torchrun with two or more ranks")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    e = abi.Engine(local)
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(abi.tp_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    e.tp_init(bytes(uid.cpu().numpy()), rank, world)
    for tokens in args.tokens:
        count = tokens * args.d
        row, st = [], None
        for own in (True, False):
            t, s = e.tp_allreduce_timed(count, args.iters, own)
            st = s if own else st
            ms = torch.tensor([t], device="cuda")
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            row.append(float(ms.item()))
        if rank == 0:
            mb = count * 2 / 1e6
            bus = lambda ms: 2 * (world - 1) / world * count * 2 / (ms / 1e3) / 1e9  # ring-equivalent GB/s
            print(f"all-reduce w={world} [{tokens} x {args.d}] bf16 {mb:.2f} MB: own {1e3 * row[0]:.1f} us "
                  f"({bus(row[0]):.0f} GB/s bus), nccl {1e3 * row[1]:.1f} us ({bus(row[1]):.0f} GB/s bus)")
            rel = [(x - st[0]) / 1e3 if x else float("nan") for x in st[:7]]
            print(f"  own, one call on rank 0 (us from CTA 0's entry): dependency {rel[1]:.1f}, partials ready "
                  f"{rel[2]:.1f}, share reduced {rel[3]:.1f}, last CTA {rel[6]:.1f}, shares ready {rel[4]:.1f}, "
                  f"end {rel[5]:.1f}")
    e.close()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    a = sub.add_parser("attention")
    a.add_argument("--dh", type=int, default=128)
    a.add_argument("--group", type=int, default=4)
    a.add_argument("--kv-heads", type=int, default=8)
    a.add_argument("--seqs", type=int, default=32)
    a.add_argument("--new", type=int, default=6)
    a.add_argument("--steps", type=int, default=3)
    a.add_argument("--ctx-lo", type=int, default=512)
    a.add_argument("--ctx-hi", type=int, default=2048)
    a.add_argument("--stamps", action="store_true", help="per-CTA phase stamps of the last attention launch")
    sp = sub.add_parser("sampler")
    sp.add_argument("--seqs", type=int, default=32)
    sp.add_argument("--k", type=int, default=5)
    sp.add_argument("--vocab", type=int, default=128256)
    sp.add_argument("--temperature", type=float, default=0.8)
    sp.add_argument("--steps", type=int, default=3)
    sp.add_argument("--logit-std", type=float, default=2.0,
                    help="std of the synthetic N(0, s^2) logits (small: near-uniform rows, as from random-init models)")
    f = sub.add_parser("forward")
    f.add_argument("--shape", choices=sorted(FWD_SHAPES), default="draft")
    f.add_argument("--layers", type=int, default=4)
    f.add_argument("--seqs", type=int, default=32)
    f.add_argument("--steps", type=int, default=3)
    g = sub.add_parser("gemm")
    g.add_argument("--n", type=int, default=28672)
    g.add_argument("--k", type=int, default=4096)
    g.add_argument("--m", type=int, default=192)
    g.add_argument("--reps", type=int, default=3)
    ar = sub.add_parser("allreduce")
    ar.add_argument("--tokens", type=int, nargs="+", default=[16, 80, 128, 640])
    ar.add_argument("--d", type=int, default=8192)
    ar.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    {"attention": attention, "sampler": sampler, "gemm": gemm, "forward": forward, "allreduce": allreduce}[args.case](args)


if __name__ == "__main__":
    main()
