"""qkv_part_rope config callables: N(0,1) bf16 qkv from a seeded CPU generator and the standard
rotary table (inverse frequencies 10000^(-2i/rope_dim), positions 0..S-1) in fp32; the checker is
``references.qkv_part_rope_ref``."""

from __future__ import annotations

import torch

from kernel_opt_agent_b200 import references

KERNEL_OPT_CHARACTERISTICS = {
    "is_matmul_like": False,
    "supports_tensor_core_candidate": False,
    "memory_bound": True,
}


def input_generator(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> dict:  # noqa: ARG001
    from kernel_opt_agent_b200.qkv_part_rope import get_inputs
    return get_inputs(batch=int(size["batch"]), seq_len=int(size["seq_len"]), q_heads=int(size["q_heads"]),
                      kv_heads=int(size["kv_heads"]), head_dim=int(size["head_dim"]),
                      nope_dim=int(size["nope_dim"]), seed=seed, device=device)


def reference_fn(inputs: dict) -> torch.Tensor:
    return references.qkv_part_rope_ref(**inputs)


def flops_fn(size: dict) -> int:
    rope = int(size["head_dim"]) - int(size["nope_dim"])
    return int(size["batch"]) * int(size["seq_len"]) * (int(size["q_heads"]) + int(size["kv_heads"])) * rope * 6


def bytes_fn(size: dict, dtype: torch.dtype) -> int:  # noqa: ARG001
    """qkv read and written in bf16, the cos and sin tables read once."""
    b, s = int(size["batch"]), int(size["seq_len"])
    heads = int(size["q_heads"]) + 2 * int(size["kv_heads"])
    d, nope = int(size["head_dim"]), int(size["nope_dim"])
    return b * s * heads * d * 2 * 2 + s * ((d - nope) // 2) * 4 * 2
