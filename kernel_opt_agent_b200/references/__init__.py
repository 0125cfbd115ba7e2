"""Correctness references for the harness (mirror of the reference's ``references/``).

These are the checkers ``kernel_configs/*.reference_fn`` call, as in the reference
(``references/__init__.py:7-23``).  They are plain PyTorch on the inputs' device and never part
of a kernel_fn call.
"""

from .flash_attention_2 import flash_attention_2_ref
from .qkv_part_rope import qkv_part_rope_ref
from .qwen35moe_gdn_prefill import qwen35moe_gdn_prefill_ref
from .rms_norm import rms_norm_ref
from .swiglu_input_quant import swiglu_input_quant_ref

__all__ = ["flash_attention_2_ref", "qkv_part_rope_ref", "qwen35moe_gdn_prefill_ref", "rms_norm_ref",
           "swiglu_input_quant_ref"]
