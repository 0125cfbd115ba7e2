"""swiglu_input_quant plugin module (the harness's ``kernel_configs/swiglu_input_quant.*`` op,
checked by ``references/swiglu_input_quant.py:6-30``): ``kernel_fn(x, eps=1e-15)`` with
x [M, 2N] bf16 = [x0 | x1] returns (out [M, N] bf16 = x0 * silu(x1), x_fp8 [M, 2N] e4m3 with
per-row 128-column-block scales, x_scale [2N / 128, M] fp32); runs ``tokmix_swiglu_input_quant``
(``csrc/neighbour_ops.cu``), no fallback."""

from __future__ import annotations

import torch

from . import _lib

KERNEL_TYPE = "swiglu_input_quant"


def kernel_fn(x: torch.Tensor, eps: float = 1e-15):
    if x.dtype != torch.bfloat16 or x.ndim != 2 or not x.is_cuda:
        raise ValueError("x must be a 2-D bfloat16 CUDA tensor [M, 2N]")
    m, two_n = x.shape
    if two_n % 256 != 0:
        raise ValueError("the last dimension of x (2N) must be a multiple of 256")
    n = two_n // 2
    x = x.contiguous()
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    x_fp8 = torch.empty((m, two_n), dtype=torch.float8_e4m3fn, device=x.device)
    x_scale = torch.empty((two_n // 128, m), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().tokmix_swiglu_input_quant(x.data_ptr(), out.data_ptr(), x_fp8.data_ptr(), x_scale.data_ptr(),
                                                   m, n, float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "swiglu_input_quant")
    return out, x_fp8, x_scale


def get_inputs(M: int = 4096, N: int = 7168, seed: int = 42, device: str = "cuda") -> dict:
    gen = torch.Generator().manual_seed(seed)
    return {"x": torch.randn(M, 2 * N, generator=gen).to(torch.bfloat16).to(device)}


def get_flops(M: int = 4096, N: int = 7168) -> int:
    return 13 * M * N


def get_bytes(M: int = 4096, N: int = 7168, element_size: int = 2) -> int:
    return M * N * 2 * element_size + M * N * element_size + M * N * 2 + (2 * N // 128) * M * 4
