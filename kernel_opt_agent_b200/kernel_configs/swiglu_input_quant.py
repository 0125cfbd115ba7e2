"""swiglu_input_quant config callables: N(0,1) x [M, 2N] from a seeded CPU generator; the checker
is ``references.swiglu_input_quant_ref``."""

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
    return {"x": torch.randn(m, 2 * n, generator=gen).to(dtype).to(device)}


def reference_fn(inputs: dict):
    return references.swiglu_input_quant_ref(inputs["x"])


def flops_fn(size: dict) -> int:
    return 13 * int(size["M"]) * int(size["N"])


def bytes_fn(size: dict, dtype: torch.dtype) -> int:
    """x read, out written, x_fp8 written (1 byte), the fp32 scales written."""
    m, n = int(size["M"]), int(size["N"])
    eb = dtype_bytes(dtype)
    return m * 2 * n * eb + m * n * eb + m * 2 * n + (2 * n // 128) * m * 4
