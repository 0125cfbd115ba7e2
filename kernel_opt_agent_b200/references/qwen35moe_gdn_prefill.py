"""Reference for qwen35moe_gdn_prefill: the fp32 token-by-token recurrence of the reference's
scalar kernel ``kernels/qwen35moe_gdn_prefill.cu:55-99`` (called by the reference's
``references/qwen35moe_gdn_prefill.py:10-19``), written with PyTorch ops batched over
(sequence, head) so it runs on the inputs' device.  Value head h reads key head h % Hk."""

from __future__ import annotations

import torch


def qwen35moe_gdn_prefill_ref(q, k, v, g, beta, state=None, scale=None, cu_seqlens=None):
    D = q.shape[-1]
    if scale is None:
        scale = D ** -0.5
    hk, hv = q.shape[2], v.shape[2]
    dev = q.device
    qf, kf, vf = (t.to(torch.float32) for t in (q, k, v))
    gf, bf = g.to(torch.float32), beta.to(torch.float32)
    head_map = torch.arange(hv, device=dev) % hk
    if cu_seqlens is None:
        B, T = q.shape[0], q.shape[1]
        segments = [(b, 0, T) for b in range(B)]
    else:
        cu = [int(x) for x in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
        segments = [(0, cu[i], cu[i + 1]) for i in range(len(cu) - 1)]
    out = torch.empty(v.shape, dtype=torch.float32, device=dev)
    finals = []
    for n, (b, t0, t1) in enumerate(segments):
        S = (state[n].to(torch.float32).clone() if state is not None
             else torch.zeros(hv, vf.shape[-1], D, device=dev))
        for t in range(t0, t1):
            kt = kf[b, t][head_map]                      # [hv, D]
            qt = qf[b, t][head_map]
            gam = torch.exp(gf[b, t])[:, None, None]      # [hv,1,1]
            kv = torch.einsum("hck,hk->hc", S, kt)
            delta = (vf[b, t] - gam[:, :, 0] * kv) * bf[b, t][:, None]
            S = gam * S + delta[:, :, None] * kt[:, None, :]
            out[b, t] = torch.einsum("hck,hk->hc", S, qt) * scale
        finals.append(S)
    return [out.to(v.dtype), torch.stack(finals)]
