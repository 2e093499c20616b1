"""yk_spec_verify_logits_noalloc: verification for hosts that cannot allocate.

Some hosts own all device memory themselves -- a serving loop that hands every
free byte of HBM to its own arenas at start-up -- so no call may cudaMalloc
behind their back.  This entry point works only on buffers the caller passes in
plus a fixed static scratch array.  The test checks, through the C-ABI, that two
calls in a row (different inputs, sharing that scratch) give exactly the tokens
and counts of the allocating entry point (yk_spec_sample_logits: the same
statistics and verification kernels), that a draft token outside the vocabulary
only marks its sequence (count -1) and is never used as an index, and that an
oversized batch is refused.  Device buffers come from torch (plumbing only).
This file is named so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu


def _case(seed, B, k, V):
    rng = np.random.default_rng(seed)
    dl = rng.normal(0, 2.0, (B, k, V)).astype(np.float32)
    tl = rng.normal(0, 2.0, (B, k + 1, V)).astype(np.float32)
    return dl, tl, np.arange(100, 100 + B, dtype=np.uint32)


def test_noalloc_verify_matches_allocating_entry(engine):
    import torch

    B, k, V = 6, 4, 50000
    cases = [(_case(1, B, k, V), 0.8, 11, 3), (_case(2, B, k, V), 1.0, 12, 4)]
    # Reference results and draft probabilities from the allocating entry point.
    expected = []
    s = abi.Sampler(engine, B, k, V)
    try:
        for (dl, tl, ids), T, seed, step in cases:
            drafts, out, cnt = s.sample_logits(dl, tl, T, seed, step, ids)
            p = np.stack([np.stack([s.read_probs(b, j) for j in range(k)]) for b in range(B)])
            expected.append((tl, p, drafts, ids, out, cnt))
    finally:
        s.close()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    bufs = []
    for (tl, p, drafts, ids, _, _), (_, T, seed, step) in zip(expected, cases):
        b = dict(tl=torch.from_numpy(tl).to(dev), p=torch.from_numpy(p).to(dev),
                 d=torch.from_numpy(drafts.view(np.int32)).to(dev), ids=torch.from_numpy(ids.view(np.int32)).to(dev),
                 out=torch.full((B, k + 1), -1, dtype=torch.int32, device=dev),
                 cnt=torch.full((B,), -1, dtype=torch.int32, device=dev), T=T, seed=seed, step=step)
        bufs.append(b)
    fn = abi.lib().yk_spec_verify_logits_noalloc
    for b in bufs:  # two calls in a row on one stream, sharing the static scratch
        abi.check(fn(0, C.c_void_p(stream.cuda_stream), b["tl"].data_ptr(), b["p"].data_ptr(), b["d"].data_ptr(),
                     b["ids"].data_ptr(), B, k, V, b["T"], b["seed"], b["step"], b["out"].data_ptr(),
                     b["cnt"].data_ptr()))
    stream.synchronize()
    for b, (_, _, _, _, out, cnt) in zip(bufs, expected):
        got_cnt = b["cnt"].cpu().numpy()
        got_out = b["out"].cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(got_cnt, cnt)
        for i in range(B):
            assert got_out[i, : cnt[i]].tolist() == out[i, : cnt[i]].tolist()
    # A draft token >= V (sequence 2): that sequence is marked, the others unchanged.
    b = bufs[0]
    bad = b["d"].clone()
    bad[2, 1] = V
    cnt2 = torch.full((B,), -7, dtype=torch.int32, device=dev)
    abi.check(fn(0, C.c_void_p(stream.cuda_stream), b["tl"].data_ptr(), b["p"].data_ptr(), bad.data_ptr(),
                 b["ids"].data_ptr(), B, k, V, b["T"], b["seed"], b["step"], b["out"].data_ptr(), cnt2.data_ptr()))
    stream.synchronize()
    exp_cnt = expected[0][5].copy()
    exp_cnt[2] = -1
    np.testing.assert_array_equal(cnt2.cpu().numpy(), exp_cnt)
    # Larger than the fixed scratch: refused before anything is launched.
    big = bufs[0]
    st = fn(0, C.c_void_p(stream.cuda_stream), big["tl"].data_ptr(), big["p"].data_ptr(), big["d"].data_ptr(),
            big["ids"].data_ptr(), 4096, 4, V, 1.0, 1, 1, big["out"].data_ptr(), big["cnt"].data_ptr())
    assert st == abi.YK_ERR_ARG and "exceed" in abi.last_error()
