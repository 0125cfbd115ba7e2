"""B200-native (sm_100a) prefill token mixers behind the kernel_opt_agent plugin contract.

Plugin modules (drop-ins for the reference's ``kernels_optimized/<name>.py``):
  * :mod:`kernel_opt_agent_b200.flash_attention_2`     -- causal attention forward
  * :mod:`kernel_opt_agent_b200.qwen35moe_gdn_prefill` -- chunked gated-delta-rule prefill

Both call the hand-written tcgen05/TMA kernels in ``libtokmix.so`` through the C ABI in
``include/tokmix.h``.  ``kernel_configs`` and ``references`` mirror the reference's registry and
checkers; ``sharding`` holds the multi-GPU work partition.
"""

from . import flash_attention_2, qwen35moe_gdn_prefill  # noqa: F401

__all__ = ["flash_attention_2", "qwen35moe_gdn_prefill"]
