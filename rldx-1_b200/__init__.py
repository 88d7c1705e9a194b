"""B200-native (sm_100a) MSAT real-time inference: the action heads of RLDX-1, plus the
VLM-backbone prefill and memory module that feed them in batched serving.

  rldx_b200.chain.B200ExpandedActionHeadChain   drop-in for CustomExpandedActionHeadChain
  rldx_b200.chain.B200ActionHeadChain           drop-in for CustomActionHeadChain (no add-ons)
  rldx_b200.block.B200ExpandedDoubleStreamBlock one joint block (ExpandedDoubleStreamBlock)
  rldx_b200.llm.B200LLMChain                    drop-in for CustomLLMChain (Qwen3 decoder prefill)
  rldx_b200.llm.B200MemoryChain                 drop-in for CustomMemoryChain (TransformerMemory)
  rldx_b200.llm.B200MemoryCache                 GraphSafeVLA's memory window + _process_memory
  rldx_b200.serve.apply_optimization            installs the native head behind model.get_action
  rldx_b200.torch_ops                           torch.ops.b200msat.* (the reference's ds::/ss:: ops)
  rldx_b200.ops                                 per-kernel wrappers (tests, op-level use)
  rldx_b200.replicas                            data-parallel replicas (one process per GPU)
  rldx_b200.microbench                          config-1 / 3 / 4 / VLM-prefill measurements

Everything computes in librldx_b200.so (hand-written sm_100a kernels behind a C ABI,
include/rldx_b200.h).  There is no CPU or library fallback.
"""

from ._lib import RldxError, load  # noqa: F401

__all__ = ["RldxError", "load"]
