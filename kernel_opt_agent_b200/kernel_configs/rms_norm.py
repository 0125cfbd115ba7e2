"""rms_norm config callables: N(0,1) x and weight from a seeded CPU generator; the checker is
``references.rms_norm_ref``."""

from __future__ import annotations

import torch

from kernel_opt_agent_b200 import references
from ._utils import dtype_bytes

KERNEL_OPT_CHARACTERISTICS = {
    "is_matmul_like": False,
    "supports_tensor_core_candidate": False,
    "memory_bound": True,
}


def input_generator(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> dict:
    gen = torch.Generator().manual_seed(seed)
    m, n = int(size["M"]), int(size["N"])
    return {"x": torch.randn(m, n, generator=gen).to(dtype).to(device),
            "weight": torch.randn(n, generator=gen).to(dtype).to(device)}


def reference_fn(inputs: dict) -> torch.Tensor:
    return references.rms_norm_ref(inputs["x"], inputs["weight"])


def flops_fn(size: dict) -> int:
    return 6 * int(size["M"]) * int(size["N"])


def bytes_fn(size: dict, dtype: torch.dtype) -> int:
    """x read, out written, weight read once."""
    m, n = int(size["M"]), int(size["N"])
    return (2 * m * n + n) * dtype_bytes(dtype)
