"""qwen35moe_gdn_decode config callables: the prefill's random workload with seq_len = 1 and
per-sequence N(0, state_std) states (default 0.02); the checker is the prefill reference, whose
token loop is the decode step (``kernels/qwen35moe_gdn_prefill.cu:55-99``)."""

from __future__ import annotations

import torch

from kernel_opt_agent_b200 import references
from ._utils import dtype_bytes
from .qwen35moe_gdn_prefill import D, H_K, H_V, random_inputs

KERNEL_OPT_CHARACTERISTICS = {
    "is_matmul_like": False,
    "supports_tensor_core_candidate": False,
    "memory_bound": True,
}


def input_generator(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> dict:
    return random_inputs(int(size["batch"]), 1, dtype, device, seed=seed,
                         state_std=float(size.get("state_std", 0.02)))


def reference_fn(inputs: dict) -> list[torch.Tensor]:
    return references.qwen35moe_gdn_prefill_ref(**inputs)


def flops_fn(size: dict) -> int:
    """The reference's recurrent count for one token per sequence."""
    return 4 * H_V * int(size["batch"]) * D * D


def bytes_fn(size: dict, dtype: torch.dtype) -> int:
    """The reference's byte formula for one token per sequence, one element size."""
    b = int(size["batch"])
    return (2 * b * H_K * D + 2 * b * H_V * D + 2 * b * H_V + 2 * b * H_V * D * D) * dtype_bytes(dtype)
