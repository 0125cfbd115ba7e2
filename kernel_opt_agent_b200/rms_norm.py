"""rms_norm plugin module (the harness's ``kernel_configs/rms_norm.*`` op, checked by
``references/rms_norm.py:6-10``): ``kernel_fn(x, weight, eps=1e-6) -> out``,
out = x / sqrt(mean(x^2, last dim) + eps) * weight in fp32, returned in x's dtype (bf16 or fp16);
runs ``tokmix_rms_norm`` (``csrc/neighbour_ops.cu``), no fallback."""

from __future__ import annotations

import torch

from . import _lib

KERNEL_TYPE = "rms_norm"
_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16}


def kernel_fn(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if x.dtype not in _DTYPES or weight.dtype != x.dtype:
        raise ValueError("x and weight must both be bfloat16 or both float16")
    if not x.is_cuda or weight.device != x.device:
        raise ValueError("x and weight must be CUDA tensors on one device")
    n = x.shape[-1]
    if tuple(weight.shape) != (n,) or n % 8 != 0:
        raise ValueError("weight must be [N] with N (the last dimension of x) a multiple of 8")
    x = x.contiguous()
    w = weight.contiguous()
    out = torch.empty_like(x)
    rows = x.numel() // n
    with torch.cuda.device(x.device):
        rc = _lib.load().tokmix_rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, n, _DTYPES[x.dtype],
                                         float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "rms_norm")
    return out


def get_inputs(M: int = 2048, N: int = 4096, dtype: torch.dtype = torch.bfloat16, seed: int = 42,
               device: str = "cuda") -> dict:
    gen = torch.Generator().manual_seed(seed)
    return {"x": torch.randn(M, N, generator=gen).to(dtype).to(device),
            "weight": torch.randn(N, generator=gen).to(dtype).to(device)}


def get_flops(M: int = 2048, N: int = 4096) -> int:
    return 6 * M * N


def get_bytes(M: int = 2048, N: int = 4096, element_size: int = 2) -> int:
    return (2 * M * N + N) * element_size
