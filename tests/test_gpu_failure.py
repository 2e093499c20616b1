"""Failure detection on the device, without faulting the GPU.

Every wait inside this module's kernels is bounded: when it gives up, the kernel
records YK_DEV_ERR_TIMEOUT in the engine's error word and returns, and the host
call reports YK_ERR_TIMEOUT.  Here a kernel waits, with the same bounded wait,
on a barrier that nothing ever arrives at; the call must end with
YK_ERR_TIMEOUT after about the budget, the error word must be cleared, and the
same engine must then run a normal verify step that matches the oracle.
(The host-side failures -- a rank that never joins, a rank that leaves -- are
in test_gpu_tp.py; the scheduler's host logic is tested on the CPU.)
"""
import numpy as np
import pytest

from helpers import TINY, PageTables, forward_pair, gpu_model, oracle_twin
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_engine_stays_usable(engine, oracle):
    st, waited = engine.wait_timeout(50)
    assert st == abi.YK_ERR_TIMEOUT, abi.last_error()
    assert 50.0 <= waited < 1000.0
    assert engine.device_error() == 0  # reported once, then cleared
    m, pool = gpu_model(engine, TINY, abi.DTYPE_BF16, seed=3, num_blocks=16)
    try:
        orc = oracle_twin(oracle, m, TINY, 16, emulate_bf16=True, nthreads=4)
        rng = np.random.default_rng(0)
        g, o = forward_pair(m, pool, orc, PageTables(16), [(0, rng.integers(0, 512, 21).tolist(), 0),
                                                           (1, rng.integers(0, 512, 6).tolist(), 0)])
        assert np.abs(g - o).max() / np.abs(o).max() < 2e-2
        assert engine.device_error() == 0
    finally:
        pool.close()
        m.close()
