"""Reference for qkv_part_rope (``references/qkv_part_rope.py:6-45``): the first q_heads + kv_heads
heads of qkv [B, S, H, D] get their last D - nope_dim columns rotated (pairs (j, j + half), fp32),
the remaining (value) heads and the nope columns are copied."""

from __future__ import annotations

import torch


def qkv_part_rope_ref(qkv, cos, sin, q_heads: int = 10, kv_heads: int = 1, nope_dim: int = 192,
                      negative_sin: bool = False, **kwargs) -> torch.Tensor:
    if qkv.dim() == 3:
        qkv = qkv.unsqueeze(0)
    half = (qkv.shape[-1] - nope_dim) // 2
    nrot = q_heads + kv_heads
    out = qkv.clone()
    rope = qkv[:, :, :nrot, nope_dim:].to(torch.float32)            # [B, S, nrot, 2 half]
    x0, x1 = rope[..., :half], rope[..., half:]
    c = cos.to(torch.float32)[None, :, None, :]
    s = sin.to(torch.float32)[None, :, None, :] * (-1.0 if negative_sin else 1.0)
    out[:, :, :nrot, nope_dim:nope_dim + half] = (x0 * c - x1 * s).to(qkv.dtype)
    out[:, :, :nrot, nope_dim + half:] = (x0 * s + x1 * c).to(qkv.dtype)
    return out
