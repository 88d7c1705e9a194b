"""B200-native (sm_100a) MSAT real-time inference: the all-modality action head of RLDX-1.

  rldx_b200.chain.B200ExpandedActionHeadChain   drop-in for CustomExpandedActionHeadChain
  rldx_b200.ops                                 per-kernel wrappers (tests, op-level use)
  rldx_b200.replicas                            data-parallel replicas (one process per GPU)

Everything computes in librldx_b200.so (hand-written sm_100a kernels behind a C ABI,
include/rldx_b200.h).  There is no CPU or library fallback.
"""

from ._lib import RldxError, load  # noqa: F401

__all__ = ["RldxError", "load"]
