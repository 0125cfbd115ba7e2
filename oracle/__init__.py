"""The oracle -- TEST INFRASTRUCTURE ONLY.

CPU restatements of the two token-mixer kernels' reference maths, used as the parity checker by
``tests/``, by ``__graft_entry__.smoke()`` and by the CPU-baseline leg of ``bench.py``.  Nothing
in the product package imports this module; the CUDA library never calls it.

* ``fa2_attention``        -- restates ``references/flash_attention_2.py:27-41``: the reference
  delegates to ``torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal,
  scale=sm_scale)`` (torch 2.11.0, ``uv.lock:580-581``).  Here: fp32
  ``softmax(q k^T * scale + causal_mask) v`` with the top-left-aligned causal mask SDPA uses,
  and grouped-query heads mapped as SDPA's ``enable_gqa`` does (q head h reads kv head
  ``h // (Hq // Hkv)``).
* ``gdn_recurrent``        -- the C restatement in ``gdn_recurrent.c`` of the reference's fp32
  scalar recurrence ``kernels/qwen35moe_gdn_prefill.cu:31-100``, called through ctypes.
* ``gdn_recurrent_numpy``  -- the same recurrence written with numpy row operations (a second,
  independent transcription used to cross-check the C code on small cases).
* ``gdn_chunked_numpy``    -- the chunked (WY / UT-transform) form of the same maths in float64,
  an independent algorithm that must agree with the recurrence to rounding.

Parity pins (see ``tests/test_oracle.py``): the FA2 restatement is checked against torch's own
SDPA run in this container; the GDN restatement is checked against outputs of the reference's
own scalar CUDA kernel (built from the reference sources by ``oracle/build_ref.py`` and run on a
B200), stored under ``tests/golden/``.
"""

from __future__ import annotations

import ctypes
import math
import os
import pathlib

import numpy as np

_HERE = pathlib.Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libgdn_oracle.so"
_lib = None


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            from . import build as _build

            _build.build_oracle()
        lib = ctypes.CDLL(str(_LIB_PATH))
        f = lib.oracle_gdn_recurrent
        f.restype = ctypes.c_int
        fp = ctypes.POINTER(ctypes.c_float)
        f.argtypes = [fp, fp, fp, fp, fp, fp, fp, fp, ctypes.POINTER(ctypes.c_int64), ctypes.c_int, ctypes.c_int,
                      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def gdn_recurrent(q, k, v, g, beta, state=None, scale=None, cu_seqlens=None, nthreads: int | None = None):
    """fp32 gated-delta-rule recurrence (reference ``gdn_ref_kernel``).

    Batched layout (``cu_seqlens is None``): q, k [B,T,Hk,Dk]; v [B,T,Hv,Dv]; g, beta [B,T,Hv];
    state [B,Hv,Dv,Dk] or None.  Varlen layout: q, k [1,Ttot,Hk,Dk] (or [Ttot,Hk,Dk]) etc. with
    cu_seqlens [N+1] and state [N,Hv,Dv,Dk].  Returns (out like v, final_state [N,Hv,Dv,Dk]).
    """
    q = _f32(q)
    k = _f32(k)
    v = _f32(v)
    g = _f32(g)
    beta = _f32(beta)
    if cu_seqlens is None:
        B, T, hk, dk = q.shape
        cu = np.arange(B + 1, dtype=np.int64) * T
    else:
        cu = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int64))
        hk, dk = q.shape[-2], q.shape[-1]
    nseq = cu.shape[0] - 1
    hv, dv = v.shape[-2], v.shape[-1]
    if scale is None:
        scale = dk ** -0.5
    st_in = None if state is None else _f32(state)
    out = np.empty_like(v)
    st_out = np.empty((nseq, hv, dv, dk), dtype=np.float32)
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    rc = _load().oracle_gdn_recurrent(
        _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(st_in) if st_in is not None else None, _ptr(out),
        _ptr(st_out), cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), int(nseq), int(hk), int(hv), int(dk),
        int(dv), float(scale), int(nthreads))
    if rc != 0:
        raise ValueError("oracle_gdn_recurrent rejected its arguments")
    if cu_seqlens is None:
        st_out = st_out.reshape(q.shape[0], hv, dv, dk)
    return out, st_out


def l2norm_rows(x, eps: float = 1e-6) -> np.ndarray:
    """x / sqrt(sum(x^2, last axis) + eps) in fp32: the q/k normalisation the workloads apply
    before the reference's GDN kernel (which takes normalised q, k:
    ``kernels/qwen35moe_gdn_prefill.py:107-136``), restated for the ``qk_l2norm`` option."""
    x = _f32(x)
    return (x / np.sqrt((x * x).sum(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))).astype(np.float32)


def gdn_gates(a, b, a_log, dt_bias):
    """The Qwen3.5 gated-delta-net gates from the raw projections, in fp32:
    g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b) (A_log, dt_bias per value head, the
    last axis); restated for the ``gates`` option (the reference takes g and beta ready-made)."""
    a, b = _f32(a), _f32(b)
    x = a + _f32(dt_bias)
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)
    g = (-np.exp(_f32(a_log)) * sp).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
    return g, beta


def gdn_recurrent_numpy(q, k, v, g, beta, state=None, scale=None):
    """Row-vectorised numpy transcription of ``kernels/qwen35moe_gdn_prefill.cu:55-99`` (batched
    layout only; small cases).  fp32 throughout."""
    q = _f32(q)
    k = _f32(k)
    v = _f32(v)
    g = _f32(g)
    beta = _f32(beta)
    B, T, hk, dk = q.shape
    hv, dv = v.shape[2], v.shape[3]
    if scale is None:
        scale = dk ** -0.5
    scale = np.float32(scale)
    out = np.zeros_like(v)
    S_all = np.zeros((B, hv, dv, dk), np.float32) if state is None else _f32(state).copy()
    for b in range(B):
        for h in range(hv):
            kh = h % hk
            S = S_all[b, h]
            for t in range(T):
                kt = k[b, t, kh]
                gam = np.float32(math.exp(float(g[b, t, h])))
                kv = S @ kt
                delta = (v[b, t, h] - gam * kv) * beta[b, t, h]
                S = gam * S + delta[:, None] * kt[None, :]
                out[b, t, h] = (S @ q[b, t, kh]) * scale
            S_all[b, h] = S
    return out, S_all


def gdn_chunked_numpy(q, k, v, g, beta, state=None, scale=None, chunk: int = 64):
    """Chunked (UT / WY) form of the same recurrence, float64, batched layout.

    Per chunk of C tokens with in-chunk cumulative log-decay G_t and incoming state S0 ([v][k]):
        L_ts   = exp(G_t - G_s) (k_t . k_s)            for s < t
        T      = (I + diag(beta) L)^-1 diag(beta)
        Delta  = T V - T diag(e^G) K S0^T
        O      = scale * (diag(e^G) Q S0^T + M Delta), M_ts = exp(G_t - G_s)(q_t . k_s), s <= t
        S_C    = e^{G_C} S0 + (diag(e^{G_C - G}) Delta)^T K
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    g = np.asarray(g, np.float64)
    beta = np.asarray(beta, np.float64)
    B, T, hk, dk = q.shape
    hv, dv = v.shape[2], v.shape[3]
    if scale is None:
        scale = dk ** -0.5
    out = np.zeros((B, T, hv, dv))
    S_all = np.zeros((B, hv, dv, dk)) if state is None else np.asarray(state, np.float64).copy()
    for b in range(B):
        for h in range(hv):
            kh = h % hk
            S = S_all[b, h]
            for c0 in range(0, T, chunk):
                c1 = min(T, c0 + chunk)
                K = k[b, c0:c1, kh]
                Q = q[b, c0:c1, kh]
                V = v[b, c0:c1, h]
                G = np.cumsum(g[b, c0:c1, h])
                bt = beta[b, c0:c1, h]
                n = c1 - c0
                dec = np.exp(np.minimum(G[:, None] - G[None, :], 0.0))
                tri_strict = np.tril(np.ones((n, n)), -1)
                tri = np.tril(np.ones((n, n)))
                L = dec * (K @ K.T) * tri_strict
                Tm = np.linalg.solve(np.eye(n) + bt[:, None] * L, np.diag(bt))
                eG = np.exp(G)
                Delta = Tm @ V - Tm @ (eG[:, None] * K) @ S.T
                M = dec * (Q @ K.T) * tri
                out[b, c0:c1, h] = scale * ((eG[:, None] * Q) @ S.T + M @ Delta)
                S = np.exp(G[-1]) * S + (np.exp(G[-1] - G)[:, None] * Delta).T @ K
            S_all[b, h] = S
    return out, S_all


def fa2_attention(q, k, v, causal: bool = True, sm_scale: float | None = None, dtype=np.float32):
    """softmax(q k^T * scale + mask) v for q [B,Hq,S,D], k/v [B,Hkv,Skv,D] (numpy arrays or
    anything convertible).  Causal mask is top-left aligned (key j visible to query i iff
    j <= i), as ``torch.nn.functional.scaled_dot_product_attention(is_causal=True)``.
    Computed in ``dtype`` (fp32 by default), returned as fp32 [B,Hq,S,D]."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    B, hq, S, D = q.shape
    hkv, skv = k.shape[1], k.shape[2]
    if hq % hkv != 0:
        raise ValueError("Hq must be a multiple of Hkv")
    group = hq // hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, hq, S, v.shape[-1]), np.float32)
    blk = 512
    for b in range(B):
        for h in range(hq):
            kk = k[b, h // group]
            vv = v[b, h // group]
            for i0 in range(0, S, blk):
                i1 = min(S, i0 + blk)
                s = (q[b, h, i0:i1] @ kk.T) * dtype(sm_scale)
                if causal:
                    rows = np.arange(i0, i1)[:, None]
                    cols = np.arange(skv)[None, :]
                    s = np.where(cols <= rows, s, -np.inf)
                m = s.max(axis=1, keepdims=True)
                p = np.exp(s - m)
                out[b, h, i0:i1] = (p @ vv) / p.sum(axis=1, keepdims=True)
    return out
