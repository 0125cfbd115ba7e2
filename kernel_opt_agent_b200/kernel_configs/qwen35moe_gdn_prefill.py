"""qwen35moe_gdn_prefill config callables.

``dist = "fixture"`` (default) reproduces the reference's deterministic inputs
(``kernel_configs/qwen35moe_gdn_prefill.py:23-44``); ``dist = "random"`` draws the B200
workload distribution from a seeded CPU generator: q, k ~ N(0,1) L2-normalised per (token,
head), v ~ N(0,1), g = -softplus(N(0,1)), beta = sigmoid(N(0,1)), zero state (or N(0, 0.02) per
sequence with ``state_std``).  ``varlen = [len, ...]`` packs sequences along T with cu_seqlens.
"""

from __future__ import annotations

import torch

from kernel_opt_agent_b200 import references
from ._utils import dtype_bytes

D = 128
H_K = 16
H_V = 32

KERNEL_OPT_CHARACTERISTICS = {
    "is_matmul_like": True,
    "supports_tensor_core_candidate": True,
    "mma_tile_m": 128,
    "effective_m": 128,
}


def _filled(shape, scale: float, bias: float, dtype: torch.dtype, device: str) -> torch.Tensor:
    n = 1
    for dim in shape:
        n *= dim
    x = torch.arange(n, dtype=torch.float32)
    x = ((x % 251) - 125.0) * scale + bias
    return x.reshape(shape).to(dtype).to(device)


def fixture_inputs(batch: int, seq_len: int, dtype: torch.dtype, device: str) -> dict:
    return {
        "q": _filled((batch, seq_len, H_K, D), 0.001, 0.0, dtype, device),
        "k": _filled((batch, seq_len, H_K, D), 0.001, 0.0, dtype, device),
        "v": _filled((batch, seq_len, H_V, D), 0.001, 0.0, dtype, device),
        "g": _filled((batch, seq_len, H_V), 0.0001, -0.01, torch.float32, device),
        "beta": _filled((batch, seq_len, H_V), 0.0001, 0.5, torch.float32, device),
        "state": _filled((batch, H_V, D, D), 0.0001, 0.0, torch.float32, device),
        "scale": D ** -0.5,
    }


def random_inputs(batch: int, seq_len: int, dtype: torch.dtype = torch.bfloat16, device: str = "cuda",
                    seed: int = 0, lengths: list[int] | None = None, state_std: float = 0.0,
                    hk: int = H_K, hv: int = H_V) -> dict:
    gen = torch.Generator().manual_seed(seed)
    if lengths is not None:
        batch, seq_len = 1, int(sum(lengths))
        nseq = len(lengths)
    else:
        nseq = batch
    q = torch.randn(batch, seq_len, hk, D, generator=gen)
    k = torch.randn(batch, seq_len, hk, D, generator=gen)
    q = q / q.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    v = torch.randn(batch, seq_len, hv, D, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(batch, seq_len, hv, generator=gen))
    beta = torch.sigmoid(torch.randn(batch, seq_len, hv, generator=gen))
    if state_std > 0:
        state = torch.randn(nseq, hv, D, D, generator=gen) * state_std
    else:
        state = torch.zeros(nseq, hv, D, D)
    out = {"q": q.to(dtype).to(device), "k": k.to(dtype).to(device), "v": v.to(dtype).to(device),
           "g": g.to(device), "beta": beta.to(device), "state": state.to(device), "scale": D ** -0.5}
    if lengths is not None:
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + int(n))
        out["cu_seqlens"] = torch.tensor(cu, dtype=torch.int32)
    return out


def varlen_lengths(n_seqs: int = 8, lo: int = 1024, hi: int = 32768, seed: int = 0) -> list[int]:
    """Sequence lengths drawn uniformly in [lo, hi] from `seed` (the packed varlen workload)."""
    gen = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n_seqs,), generator=gen)]


def input_generator(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> dict:
    if size.get("dist", "fixture") == "fixture":
        return fixture_inputs(int(size["batch"]), int(size["seq_len"]), dtype, device)
    return random_inputs(int(size["batch"]), int(size["seq_len"]), dtype, device, seed=seed,
                           lengths=size.get("varlen"), state_std=float(size.get("state_std", 0.0)))


def numerical_stability_cases(size: dict, dtype: torch.dtype, device: str, seed: int = 42) -> list[tuple[str, dict]]:
    """The reference's three cases (``kernel_configs/qwen35moe_gdn_prefill.py:47-63``) plus the
    strongly negative gate regression g ~ U(-25, -8) at T=64 recorded in the reference's
    experiment log."""
    small = dict(size)
    small["seq_len"] = min(int(small.get("seq_len", 2048)), 2048)
    small.pop("varlen", None)
    small["seq_len"] = max(small["seq_len"], 1)
    base = input_generator(small, dtype, device, seed)
    zero_state = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in base.items()}
    zero_state["state"] = torch.zeros_like(zero_state["state"])
    softer_gate = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in base.items()}
    softer_gate["g"] = torch.full_like(softer_gate["g"], -0.02)
    strong = random_inputs(1, 64, dtype, device, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1)
    strong["g"] = (torch.rand(strong["g"].shape, generator=gen) * 17.0 - 25.0).to(device)
    return [("baseline", base), ("zero_state", zero_state), ("softer_gate", softer_gate),
            ("strong_negative_gate", strong)]


def reference_fn(inputs: dict) -> list[torch.Tensor]:
    return references.qwen35moe_gdn_prefill_ref(**inputs)


def _tokens(size: dict) -> int:
    if size.get("varlen") is not None:
        return int(sum(size["varlen"]))
    return int(size["batch"]) * int(size["seq_len"])


def flops_fn(size: dict) -> int:
    """Reference recurrent count, ``kernel_configs/qwen35moe_gdn_prefill.py:70-71``."""
    return 4 * H_V * _tokens(size) * D * D


def bytes_fn(size: dict, dtype: torch.dtype) -> int:
    """Reference formula (``kernel_configs/qwen35moe_gdn_prefill.py:74-82``), one element size."""
    eb = dtype_bytes(dtype)
    tokens = _tokens(size)
    nseq = len(size["varlen"]) if size.get("varlen") is not None else int(size["batch"])
    return (2 * tokens * H_K * D + 2 * tokens * H_V * D + 2 * tokens * H_V + 2 * nseq * H_V * D * D) * eb
