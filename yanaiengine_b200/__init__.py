"""yanaiengine_b200 -- B200-native speculative draft->verify hot path of YanAIEngine.

libyk.so (include/yk.h): sm_100a kernels for the verify forward, paged
attention and the fused rejection sampler.  libyk_host.so (include/yk_host.h):
the C++ Scheduler / PagedKVCache / BlockAllocator host that drives it.
`abi` binds both through ctypes.
"""
from . import abi  # noqa: F401

__all__ = ["abi"]
