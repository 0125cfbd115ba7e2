"""Reference for flash_attention_2: ``torch.nn.functional.scaled_dot_product_attention``, as the
reference's ``references/flash_attention_2.py:11-41``, generalised to grouped-query heads
(``enable_gqa``), any head_dim, both layouts, and any device."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def flash_attention_2_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                          sm_scale: float | None = None, layout: str = "bhsd") -> torch.Tensor:
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must be 4-D")
    if layout == "bshd":
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    out = F.scaled_dot_product_attention(q.contiguous(), k.contiguous(), v.contiguous(), attn_mask=None,
                                         dropout_p=0.0, is_causal=causal, scale=float(sm_scale),
                                         enable_gqa=q.shape[1] != k.shape[1])
    if layout == "bshd":
        out = out.transpose(1, 2).contiguous()
    return out
