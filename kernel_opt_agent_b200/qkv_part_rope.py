"""qkv_part_rope plugin module (the harness's ``kernel_configs/qkv_part_rope.*`` op, checked by
``references/qkv_part_rope.py:6-45``): ``kernel_fn(qkv, cos, sin, q_heads=10, kv_heads=1,
nope_dim=192, negative_sin=False)`` with qkv [B, S, H, D] bf16 (or [S, H, D]) and cos, sin
[S, (D - nope_dim) / 2] fp32 returns a copy of qkv whose first q_heads + kv_heads heads have their
last D - nope_dim columns rotated; runs ``tokmix_qkv_part_rope`` (``csrc/neighbour_ops.cu``), no
fallback."""

from __future__ import annotations

import torch

from . import _lib

KERNEL_TYPE = "qkv_part_rope"


def kernel_fn(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, q_heads: int = 10, kv_heads: int = 1,
              nope_dim: int = 192, negative_sin: bool = False, **kwargs) -> torch.Tensor:
    if qkv.dim() == 3:
        qkv = qkv.unsqueeze(0)
    if qkv.dtype != torch.bfloat16 or qkv.dim() != 4 or not qkv.is_cuda:
        raise ValueError("qkv must be a bfloat16 CUDA tensor [batch, seq, heads, head_dim]")
    b, s, h, d = qkv.shape
    half = (d - nope_dim) // 2
    if d % 8 != 0 or nope_dim % 8 != 0 or nope_dim > d or (d - nope_dim) % 2 != 0:
        raise ValueError("head_dim and nope_dim must be multiples of 8 with nope_dim <= head_dim")
    if q_heads + kv_heads > h:
        raise ValueError("q_heads + kv_heads exceeds the number of heads")
    if tuple(cos.shape) != (s, half) or tuple(sin.shape) != (s, half):
        raise ValueError(f"cos and sin must be [{s}, {half}]")
    qkv = qkv.contiguous()
    c = cos.to(device=qkv.device, dtype=torch.float32).contiguous()
    sn = sin.to(device=qkv.device, dtype=torch.float32).contiguous()
    out = torch.empty_like(qkv)
    with torch.cuda.device(qkv.device):
        rc = _lib.load().tokmix_qkv_part_rope(qkv.data_ptr(), c.data_ptr(), sn.data_ptr(), out.data_ptr(), b, s, h, d,
                                              int(q_heads), int(kv_heads), int(nope_dim), 1 if negative_sin else 0,
                                              _lib.stream_ptr(qkv.device))
    _lib.check(rc, "qkv_part_rope")
    return out


def get_inputs(batch: int = 50, seq_len: int = 2048, q_heads: int = 10, kv_heads: int = 1, head_dim: int = 256,
               nope_dim: int = 192, seed: int = 42, device: str = "cuda") -> dict:
    gen = torch.Generator().manual_seed(seed)
    heads = q_heads + 2 * kv_heads
    rope = head_dim - nope_dim
    qkv = torch.randn(batch, seq_len, heads, head_dim, generator=gen).to(torch.bfloat16)
    inv_freq = 1.0 / (10000 ** (torch.arange(0, rope, 2, dtype=torch.float32) / rope))
    freqs = torch.outer(torch.arange(seq_len, dtype=torch.float32), inv_freq)
    return {"qkv": qkv.to(device), "cos": torch.cos(freqs).to(device), "sin": torch.sin(freqs).to(device),
            "q_heads": q_heads, "kv_heads": kv_heads, "nope_dim": nope_dim}


def get_flops(batch: int = 50, seq_len: int = 2048, q_heads: int = 10, kv_heads: int = 1, head_dim: int = 256,
              nope_dim: int = 192) -> int:
    return batch * seq_len * (q_heads + kv_heads) * (head_dim - nope_dim) * 6


def get_bytes(batch: int = 50, seq_len: int = 2048, q_heads: int = 10, kv_heads: int = 1, head_dim: int = 256,
              nope_dim: int = 192) -> int:
    return batch * seq_len * (q_heads + 2 * kv_heads) * head_dim * 2 * 2 + seq_len * ((head_dim - nope_dim) // 2) * 4 * 2
