"""Reference for swiglu_input_quant (``references/swiglu_input_quant.py:6-30``): x = [x0 | x1];
out = x0 * x1 * sigmoid(x1) (x1 in fp32, cast to x's dtype); the input x quantised to e4m3 per
128-column block with scale = max(amax, eps) / 448, the block multiplied by the scale's inverse
rounded to x's dtype before the conversion; scales as [n_blocks, M]."""

from __future__ import annotations

import torch

BLOCK = 128
E4M3_MAX = 448.0


def swiglu_input_quant_ref(x: torch.Tensor, eps: float = 1e-15):
    m, two_n = x.shape
    n = two_n // 2
    x1 = x[:, n:].to(torch.float32)
    out = (x[:, :n] * (x1 * torch.sigmoid(x1))).to(x.dtype)
    blocks = x.view(m, two_n // BLOCK, BLOCK)
    amax = blocks.to(torch.float32).abs().amax(dim=-1).clamp(min=eps)      # [m, n_blocks]
    scale = amax / E4M3_MAX
    inv = (1.0 / scale).to(x.dtype)
    x_fp8 = (blocks * inv[:, :, None]).to(torch.float8_e4m3fn).view(m, two_n)
    return out, x_fp8, scale.t().contiguous()
