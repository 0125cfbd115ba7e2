"""qwen35moe_gdn_decode plugin module -- one decode step of the Qwen3.5-MoE gated delta net, with
the module contract of the reference's plugins (``kernels/__init__.py:3-8``):

    KERNEL_TYPE, kernel_fn(q, k, v, g, beta, state, scale=None) -> [out, final_state],
    get_inputs, get_flops, get_bytes

The arguments are those of ``qwen35moe_gdn_prefill.kernel_fn`` with one token per sequence
(``kernels/qwen35moe_gdn_prefill.py:107-151`` with T = 1): q, k [B,1,Hk,128]; v [B,1,Hv,128];
g (log decay), beta [B,1,Hv]; state [B,Hv,128(v),128(k)] fp32 or None (zero); value head h reads
key head h % Hk; default scale 128**-0.5; returns [out like v, final_state fp32].  The maths is
the reference's fp32 recurrence for one token (``kernels/qwen35moe_gdn_prefill.cu:55-99``), the
step its optimised prefill special-cases for one-token chunks
(``kernels_optimized/qwen35moe_gdn_prefill.cu:865-934``).

``kernel_fn`` runs ``tokmix_gdn_decode`` (``csrc/gdn_decode.cu``); there is no fallback.  q/k/v
may be bf16 (native) or fp32 (rounded to bf16 on the device; out is then returned as fp32).
``inplace=True`` (keyword) updates ``state`` itself and returns it as final_state: a decode
loop then moves each state through HBM once per token and allocates nothing for it.
``qk_l2norm=True`` L2-normalises q and k first and ``gates=(A_log, dt_bias)`` takes raw gate
projections in place of g and beta, as in ``qwen35moe_gdn_prefill``.
"""

from __future__ import annotations

import torch

from . import _lib
from .qwen35moe_gdn_prefill import D, H_K, H_V, gdn_gates, l2norm_rows

KERNEL_TYPE = "qwen35moe_gdn_decode"


def _validate(q, k, v, g, beta, state):
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q/k/v must be [batch, 1, heads, dim]")
    if g.ndim != 3 or beta.ndim != 3:
        raise ValueError("g/beta must be [batch, 1, H_v]")
    if q.shape[1] != 1:
        raise ValueError("decode takes one token per sequence (q.shape[1] must be 1)")
    if q.shape[-1] != D or k.shape[-1] != D or v.shape[-1] != D:
        raise ValueError("head dimension must be 128")
    if q.shape != k.shape:
        raise ValueError("q and k shapes must match")
    hk, hv = q.shape[2], v.shape[2]
    if hv % hk != 0:
        raise ValueError("H_v must be a multiple of H_k")
    if v.shape[:2] != q.shape[:2] or g.shape != q.shape[:2] + (hv,) or beta.shape != g.shape:
        raise ValueError("inconsistent token/head shapes")
    tensors = [q, k, v, g, beta] + ([state] if state is not None else [])
    if any(not t.is_cuda for t in tensors):
        raise ValueError("all tensors must be CUDA tensors")
    if any(t.device != q.device for t in tensors):
        raise ValueError("all tensors must be on the same device")
    if q.dtype not in (torch.bfloat16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q/k/v must all be bfloat16 or all be float32")
    if state is not None and tuple(state.shape) != (q.shape[0], hv, D, D):
        raise ValueError(f"state shape must be [{q.shape[0]}, {hv}, 128, 128]")
    return q.shape[0], hk, hv


def kernel_fn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    state: torch.Tensor | None,
    scale: float | None = None,
    *,
    inplace: bool = False,
    qk_l2norm: bool = False,
    gates=None,
) -> list[torch.Tensor]:
    batch, hk, hv = _validate(q, k, v, g, beta, state)
    if gates is not None:
        g, beta = gdn_gates(g, beta, *gates)
    if scale is None:
        scale = D ** -0.5
    dev = q.device
    io_dtype = q.dtype
    qb = l2norm_rows(q) if qk_l2norm else q.to(torch.bfloat16).contiguous()
    kb = l2norm_rows(k) if qk_l2norm else k.to(torch.bfloat16).contiguous()
    vb = v.to(torch.bfloat16).contiguous()
    gf = g.to(torch.float32).contiguous()
    bf = beta.to(torch.float32).contiguous()
    if inplace:
        if state is None or state.dtype != torch.float32 or not state.is_contiguous():
            raise ValueError("inplace=True needs a contiguous fp32 state tensor")
        st_in = final_state = state
    else:
        st_in = state.to(torch.float32).contiguous() if state is not None else None
        final_state = torch.empty((batch, hv, D, D), dtype=torch.float32, device=dev)
    out = torch.empty(vb.shape, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.tokmix_gdn_decode(
            qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), gf.data_ptr(), bf.data_ptr(),
            st_in.data_ptr() if st_in is not None else None, final_state.data_ptr(), out.data_ptr(),
            batch, hk, hv, D, D, float(scale), _lib.DTYPE_BF16, _lib.stream_ptr(dev))
    _lib.check(rc, "qwen35moe_gdn_decode")
    if io_dtype != torch.bfloat16:
        out = out.to(io_dtype)
    return [out, final_state]


def get_inputs(batch: int = 64, dtype: torch.dtype = torch.bfloat16, seed: int = 0, device: str = "cuda",
               state_std: float = 0.02) -> dict:
    """One decode token per sequence with the B200 workload distribution (q, k L2-normalised,
    v ~ N(0,1), g = -softplus(N(0,1)), beta = sigmoid(N(0,1))) and N(0, state_std) states, drawn
    from a seeded CPU generator."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, 1, H_K, D, generator=gen)
    k = torch.randn(batch, 1, H_K, D, generator=gen)
    q = q / q.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    v = torch.randn(batch, 1, H_V, D, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(batch, 1, H_V, generator=gen))
    beta = torch.sigmoid(torch.randn(batch, 1, H_V, generator=gen))
    state = torch.randn(batch, H_V, D, D, generator=gen) * state_std
    return {"q": q.to(dtype).to(device), "k": k.to(dtype).to(device), "v": v.to(dtype).to(device),
            "g": g.to(device), "beta": beta.to(device), "state": state.to(device), "scale": D ** -0.5}


def get_flops(batch: int = 64) -> int:
    """The reference's recurrent count (``kernel_configs/qwen35moe_gdn_prefill.py:70-76``) for one token."""
    return 4 * batch * H_V * D * D


def get_bytes(batch: int = 64, element_size: int = 4) -> int:
    """The reference's byte formula (``kernel_configs/qwen35moe_gdn_prefill.py:77-82``) for one token."""
    qk = 2 * batch * H_K * D
    vo = 2 * batch * H_V * D
    gb = 2 * batch * H_V
    st = 2 * batch * H_V * D * D
    return (qk + vo + gb + st) * element_size


def algorithmic_bytes(batch: int, hk: int = H_K, hv: int = H_V) -> int:
    """Bytes one decode step must move at this library's types: q, k, v, o bf16, g, beta fp32, and
    the fp32 state read and written once."""
    return batch * (2 * hk + 2 * hv) * D * 2 + batch * 2 * hv * 4 + batch * hv * D * D * 4 * 2
