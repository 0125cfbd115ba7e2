"""flash_attention_2 config callables (the reference's ``kernel_configs/flash_attention_2.py``
semantics: RMS-normalised N(0,1) q/k, N(0,1) v, seven stability cases, reference flop/byte
formulas), extended with grouped-query heads and the [batch, seq, heads, dim] layout.  Inputs
are drawn on the CPU from a seeded generator and then moved, so every device sees the same
values."""

from __future__ import annotations

import math

import torch

from kernel_opt_agent_b200 import references
from ._utils import dtype_bytes

KERNEL_OPT_CHARACTERISTICS = {
    "is_matmul_like": True,
    "supports_tensor_core_candidate": True,
    "mma_tile_m": 128,
    "effective_m": 128,
}


def _rms_normalize(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    rms = x.square().mean(dim=-1, keepdim=True).sqrt().clamp_min(eps)
    return x / rms


def _make_attention_inputs(size: dict, dtype: torch.dtype, device: str, seed: int = 42, *, q_scale: float = 1.0,
                           k_scale: float = 1.0, v_scale: float = 1.0, rms: bool = True) -> dict:
    gen = torch.Generator().manual_seed(seed)
    b, h, s, d = size["batch"], size["head_num"], size["seq_len"], size["head_dim"]
    hkv = size.get("head_num_kv", h)
    layout = size.get("layout", "bhsd")

    def shape(nh):
        return (b, nh, s, d) if layout == "bhsd" else (b, s, nh, d)

    q = torch.randn(shape(h), generator=gen, dtype=torch.float32)
    k = torch.randn(shape(hkv), generator=gen, dtype=torch.float32)
    v = torch.randn(shape(hkv), generator=gen, dtype=torch.float32)
    if rms:
        q = _rms_normalize(q)
        k = _rms_normalize(k)
    q, k, v = q * q_scale, k * k_scale, v * v_scale
    out = {"q": q.to(dtype).to(device), "k": k.to(dtype).to(device), "v": v.to(dtype).to(device), "causal": True,
           "sm_scale": 1.0 / math.sqrt(d)}
    if layout != "bhsd":
        out["layout"] = layout
    return out


def input_generator(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> dict:
    return _make_attention_inputs(size, dtype, device, seed=seed)


def random_inputs(size: dict, dtype: torch.dtype = torch.bfloat16, device: str = "cuda", seed: int = 0) -> dict:
    """The B200 workload generator: q, k, v ~ N(0,1) from `seed` (no RMS normalisation)."""
    return _make_attention_inputs(size, dtype, device, seed=seed, rms=False)


def numerical_stability_cases(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> list[tuple[str, dict]]:
    cases = [
        ("softmax_flat", _make_attention_inputs(size, dtype, device, seed=seed, q_scale=0.5, k_scale=0.5)),
        ("softmax_nominal", _make_attention_inputs(size, dtype, device, seed=seed)),
        ("softmax_sharp", _make_attention_inputs(size, dtype, device, seed=seed, q_scale=2.0, k_scale=2.0)),
        ("qk_imbalance", _make_attention_inputs(size, dtype, device, seed=seed, q_scale=2.0, k_scale=0.5)),
        ("value_amplified", _make_attention_inputs(size, dtype, device, seed=seed, v_scale=2.0)),
    ]
    zero_q = _make_attention_inputs(size, dtype, device, seed=seed)
    zero_q["q"] = torch.zeros_like(zero_q["q"])
    cases.append(("zero_queries", zero_q))
    const_v = _make_attention_inputs(size, dtype, device, seed=seed)
    const_v["v"] = torch.full_like(const_v["v"], 0.5)
    cases.append(("constant_values", const_v))
    return cases


def reference_fn(inputs: dict) -> torch.Tensor:
    return references.flash_attention_2_ref(**inputs)


def flops_fn(size: dict) -> int:
    pairs = size["seq_len"] * (size["seq_len"] + 1) // 2
    return 4 * size["batch"] * size["head_num"] * pairs * size["head_dim"]


def bytes_fn(size: dict, dtype: torch.dtype) -> int:
    hkv = size.get("head_num_kv", size["head_num"])
    per_head = size["batch"] * size["seq_len"] * size["head_dim"] * dtype_bytes(dtype)
    return (2 * size["head_num"] + 2 * hkv) * per_head
