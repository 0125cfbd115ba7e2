"""flash_attention_2 plugin module -- drop-in for the reference's
``kernels_optimized/flash_attention_2.py`` (same module contract, ``kernels/__init__.py:3-8``):

    KERNEL_TYPE, kernel_fn(q, k, v, causal=True, sm_scale=None), get_inputs, get_flops, get_bytes

``kernel_fn`` runs the sm_100a kernel in libtokmix.so (``tokmix_fa2_fwd``); there is no fallback.
Compared with the reference module (``kernels_optimized/flash_attention_2.py:110-140``) it also
accepts grouped-query attention (k/v with fewer heads), head_dim 64 and 256 and a ``layout="bshd"``
keyword; with the reference's arguments it behaves the same: q, k, v bf16 CUDA tensors
[batch, heads, seq, head_dim], default scale 1/sqrt(head_dim), returns a new bf16 tensor.
"""

from __future__ import annotations

import math

import torch

from . import _lib

KERNEL_TYPE = "flash_attention_2"
_HEAD_DIM = 128
_HEAD_DIMS = (64, 128, 256)
_DTYPE = torch.bfloat16


def _validate_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layout: str):
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must have shape [batch, heads, seq_len, head_dim]")
    if layout not in ("bhsd", "bshd"):
        raise ValueError(f"layout must be 'bhsd' or 'bshd', got {layout!r}")
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shapes")
    hd = 1 if layout == "bhsd" else 2
    sd = 2 if layout == "bhsd" else 1
    if q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        raise ValueError("q and k/v must agree on batch and head_dim")
    if q.shape[hd] % k.shape[hd] != 0:
        raise ValueError("query heads must be a multiple of key/value heads")
    if not q.is_cuda or not k.is_cuda or not v.is_cuda:
        raise ValueError("q, k, and v must be CUDA tensors")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, and v must be on the same device")
    if q.dtype != _DTYPE or k.dtype != _DTYPE or v.dtype != _DTYPE:
        raise ValueError("q, k, and v must be bfloat16 tensors")
    if q.shape[-1] not in _HEAD_DIMS:
        raise ValueError(f"head_dim must be one of {_HEAD_DIMS}")
    return q.contiguous(), k.contiguous(), v.contiguous(), hd, sd


def kernel_fn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = True,
    sm_scale: float | None = None,
    *,
    layout: str = "bhsd",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    q, k, v, hd, sd = _validate_inputs(q, k, v, layout)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous() or out.device != q.device:
        raise ValueError("out must be a contiguous bf16 tensor shaped like q")
    lib = _lib.load()
    dev = q.device
    word = _lib.status_word(dev)
    with torch.cuda.device(dev):
        rc = lib.tokmix_fa2_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            q.shape[0], q.shape[hd], k.shape[hd], q.shape[sd], k.shape[sd], q.shape[3],
            _lib.LAYOUT_BHSD if layout == "bhsd" else _lib.LAYOUT_BSHD, 1 if causal else 0, float(sm_scale),
            word.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "flash_attention_2")
    _lib.after_launch(dev, "flash_attention_2")
    return out


def check_device_status(device: torch.device | None = None) -> None:
    """Synchronise and raise if any kernel on `device` reported a device-side timeout."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    _lib.check_status(dev, "flash_attention_2")


def get_inputs(
    batch: int = 8,
    head_num: int = 8,
    seq_len: int = 2048,
    head_dim: int = _HEAD_DIM,
    dtype: torch.dtype = _DTYPE,
    causal: bool = True,
    seed: int = 42,
    *,
    head_num_kv: int | None = None,
    layout: str = "bhsd",
    device: str = "cuda",
) -> dict:
    """N(0,1) q, k, v.  Drawn on the CPU from a seeded generator and then moved, so the same
    seed gives the same values on every device (the reference draws with torch.randn on cuda,
    ``kernels_optimized/flash_attention_2.py:143-163``)."""
    gen = torch.Generator().manual_seed(seed)
    hkv = head_num if head_num_kv is None else head_num_kv

    def shape(h):
        return (batch, h, seq_len, head_dim) if layout == "bhsd" else (batch, seq_len, h, head_dim)

    q = torch.randn(shape(head_num), generator=gen, dtype=torch.float32).to(dtype)
    k = torch.randn(shape(hkv), generator=gen, dtype=torch.float32).to(dtype)
    v = torch.randn(shape(hkv), generator=gen, dtype=torch.float32).to(dtype)
    out = {"q": q.to(device), "k": k.to(device), "v": v.to(device), "causal": causal,
           "sm_scale": 1.0 / math.sqrt(head_dim)}
    if layout != "bhsd":
        out["layout"] = layout
    return out


def get_flops(
    batch: int = 8,
    head_num: int = 8,
    seq_len: int = 2048,
    head_dim: int = _HEAD_DIM,
    causal: bool = True,
) -> int:
    """Reference formula, ``kernels_optimized/flash_attention_2.py:166-174``."""
    attn_pairs = seq_len * (seq_len + 1) // 2 if causal else seq_len * seq_len
    return 4 * batch * head_num * attn_pairs * head_dim


def get_bytes(
    batch: int = 8,
    head_num: int = 8,
    seq_len: int = 2048,
    head_dim: int = _HEAD_DIM,
    element_size: int = 2,
    *,
    head_num_kv: int | None = None,
) -> int:
    """q, k, v read once and o written once (``kernels_optimized/flash_attention_2.py:177-185``;
    with grouped-query heads k and v count ``head_num_kv`` heads)."""
    hkv = head_num if head_num_kv is None else head_num_kv
    return (2 * head_num + 2 * hkv) * batch * seq_len * head_dim * element_size
