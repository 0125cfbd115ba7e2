"""Reference for rms_norm (``references/rms_norm.py:6-10``): x scaled by the reciprocal root mean
square of its row (plus eps) and by the weight, in fp32, returned in x's dtype."""

from __future__ import annotations

import torch


def rms_norm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.to(torch.float32)
    denom = (xf.pow(2).mean(dim=-1, keepdim=True) + eps).sqrt()
    return (xf / denom * weight.to(torch.float32)).to(x.dtype)
