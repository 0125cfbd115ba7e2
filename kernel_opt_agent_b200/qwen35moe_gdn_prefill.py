"""qwen35moe_gdn_prefill plugin module -- drop-in for the reference's
``kernels_optimized/qwen35moe_gdn_prefill.py`` (module contract of ``kernels/__init__.py:3-8``):

    KERNEL_TYPE, kernel_fn(q, k, v, g, beta, state, scale=None) -> [out, final_state],
    get_inputs, get_flops, get_bytes

``kernel_fn`` runs the sm_100a chunked kernels in libtokmix.so; there is no fallback.  Three
schedules compute the same result: one CTA per (sequence, value head) doing everything
(``tokmix_gdn_prefill``, "fused"), or, when there are fewer such units than SMs, chunk-parallel
preparation of per-chunk operand records followed by one state chain per unit
(``tokmix_gdn_prefill_split``, which needs a workspace of about 73 KB per (chunk, value head),
taken from PyTorch's caching allocator): as two launches ("split"), or as one cooperative launch
whose chain CTAs consume each chunk as the preparation CTAs on the other SMs finish it
("overlap").  Argument meaning follows the reference (``kernels/qwen35moe_gdn_prefill.py:107-151``):
q, k [B,T,Hk,128]; v [B,T,Hv,128]; g (log decay), beta [B,T,Hv]; state [B,Hv,128(v),128(k)];
value head h reads key head h % Hk; default scale 128**-0.5; returns [out like v, final_state fp32].

Extensions over the reference module:
* q/k/v may be bf16 (the kernel's native type; out is then bf16).  The reference's fp32 contract
  is accepted too: fp32 q/k/v are rounded to bf16 on the device before the kernel runs and the
  output is returned as fp32.
* ``cu_seqlens`` (keyword): variable-length sequences packed along T with q.shape[0] == 1 and
  one initial state per sequence (state [N,Hv,128,128]); ``state=None`` means zero states.
* any Hk dividing Hv (the reference fixes Hk=16, Hv=32).
* ``qk_l2norm`` (keyword, default False): L2-normalise q and k per (token, head),
  ``x / sqrt(sum x^2 + 1e-6)`` in fp32, as the workloads' generators do before calling the
  reference.  bf16 q, k are normalised inside stage 1, as each chunk's rows are staged for the
  first product (the split-family schedules keep a normalised copy of k for their chains); fp32
  q, k by the separate pass ``l2norm_rows``, which also converts them to the kernels' bf16 operand.
  Both give the same bits.
* ``gates`` (keyword, default None): ``(A_log, dt_bias)`` ([Hv] each) to pass the raw gate
  projections instead of g and beta: the ``g`` and ``beta`` arguments then hold the projections
  a and b, and ``g = -exp(A_log) * softplus(a + dt_bias)``, ``beta = sigmoid(b)`` are computed on
  the device by the preparation of each chunk inside the prefill kernels (the same arithmetic as
  the separate pass ``gdn_gates``, so the results are the same bits), as Qwen3.5's GDN layer does
  before its kernel; the decode step runs the separate pass.
* ``checkpoints`` (keyword, default False): also return the state after every 64-token chunk
  as a third output -- [B, ceil(T/64), Hv, 128, 128] fp32 for a batch, [total_chunks, Hv, 128,
  128] with cu_seqlens (sequence n's chunks from ``sum(ceil(len_m/64) for m < n)``) -- for prefix
  caching or a backward pass; the last chunk's entry equals the final state.  Checkpoints come
  from the split-family schedules ("split"/"overlap", chosen whatever the unit count).
* ``mode`` (keyword): "auto" (default), "fused", "split", "overlap" or "segmented" selects the
  schedule; the environment variable TOKMIX_GDN_MODE overrides "auto".  "auto" picks "fused" when
  the units fill the SMs, else the schedule with the lowest predicted time (and the library
  itself falls back from "overlap" to two launches when the device cannot hold the cooperative
  grid).  "segmented" (``tokmix_gdn_prefill_segmented``) cuts sequences longer than a segment
  length into segments whose chains run side by side and joins them afterwards (the entry state
  of each segment enters its outputs and end state linearly); the length is the shortest whose
  chains still fit on the SMs at once, or ``segment_chunks`` (keyword, in 64-token chunks).  A batched call with one token per sequence (T = 1, the
  decode step of a serving loop) runs ``qwen35moe_gdn_decode``'s one-pass kernel instead under
  "auto" ("decode").
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

KERNEL_TYPE = "qwen35moe_gdn_prefill"
D = 128
H_K = 16
H_V = 32
# bytes; larger problems use the one-launch schedule.  75 KB per (chunk, value head): 24 GiB covers a
# batch of 16 sequences of 16384 tokens at 32 value heads (9.8 GB), an eighth of a B200's memory.
_SPLIT_MAX_WORKSPACE = 24 << 30
# Costs measured on a B200 (microseconds), from which "auto" predicts each schedule's time when
# every unit fits on the SMs at once: a chunk of the fused kernel's chain (preparation inside the
# CTA; 277 us / 32 chunks at B1 T2048, 2.9 ms / 347 chunks on a varlen slice), a chunk of the chain
# fed from prepared records (split B1 T2048: 140 us = 44 preparation + 32 chunks + gap), one
# preparation record with three preparation groups per SM (alone: 288 us for 7364 records; beside
# the chains of the overlapped launch, whose first round of records runs in lockstep: 27 us for the
# first records, 18 us each after that), the overlapped launch's start-up, and the gap between
# launches.
_US_FUSED_CHUNK = 8.5
_US_FUSED_CHUNK_WAVES = 10.2  # per chunk and unit when the units run in several waves (varlen, one GPU: 4.07 ms)
_US_CHAIN_CHUNK = 2.7
_US_PREP_RECORD = 17.5
_US_PREP_RECORD_OVERLAP = 24.0
_US_OVERLAP_START = 20.0
_US_SPLIT_GAP = 10.0
# The segmented schedule (measured launch list: B1 T2048 cut in 2, a varlen slice of 4 value
# heads cut into segments of 106 chunks): chains of a segment (start-up + per chunk), the combine
# (start-up + per extra segment of the most-cut sequence), the correction GEMM (start-up + its
# traffic: R read, out read and written, 768 B per later-segment token and head, at an effective
# 3.5 TB/s), and the gaps between its four launches.  Segments shorter than _SEG_MIN_CHUNKS are
# not made.
_US_SEG_CHAIN_START = 10.0
_US_SEG_CHAIN_CHUNK = 2.65
_US_SEG_COMBINE_START = 5.0
_US_SEG_COMBINE_STEP = 8.0
_US_SEG_CORR_START = 5.0
_SEG_CORR_BYTES_PER_US = 3.5e6
_US_SEG_GAPS = 15.0
_SEG_MIN_CHUNKS = 8
QK_L2NORM_EPS = 1e-6

_meta_cache: dict = {}


def _device_meta(lengths: tuple[int, ...], device: torch.device):
    """cu_seqlens (int32), the longest-first scheduling order and the per-sequence first chunk
    (int32, for the split schedule) with the chunk count, uploaded once per shape."""
    key = (lengths, device)
    hit = _meta_cache.get(key)
    if hit is None:
        cu, cb = [0], [0]
        for n in lengths:
            cu.append(cu[-1] + n)
            cb.append(cb[-1] + (n + 63) // 64)
        order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
        cu_t = torch.tensor(cu, dtype=torch.int32).to(device)
        order_t = torch.tensor(order, dtype=torch.int32).to(device) if len(set(lengths)) > 1 else None
        cb_t = torch.tensor(cb, dtype=torch.int32).to(device)
        hit = (cu_t, order_t, cb_t, cb[-1], cb)
        if len(_meta_cache) > 256:
            _meta_cache.clear()
        _meta_cache[key] = hit
    return hit


def _validate(q, k, v, g, beta, state, cu_seqlens):
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q/k/v must be [batch, tokens, heads, dim]")
    if g.ndim != 3 or beta.ndim != 3:
        raise ValueError("g/beta must be [batch, tokens, H_v]")
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
    if cu_seqlens is None:
        nseq = q.shape[0]
    else:
        if q.shape[0] != 1:
            raise ValueError("with cu_seqlens, q/k/v/g/beta must have batch dimension 1")
        nseq = len(cu_seqlens) - 1
        if nseq < 1:
            raise ValueError("cu_seqlens needs at least two entries")
    if state is not None and tuple(state.shape) != (nseq, hv, D, D):
        raise ValueError(f"state shape must be [{nseq}, {hv}, 128, 128]")
    return nseq, hk, hv


def _lengths(cu_seqlens, total: int) -> tuple[int, ...]:
    if isinstance(cu_seqlens, torch.Tensor):
        cu = [int(x) for x in cu_seqlens.detach().to("cpu").tolist()]
    else:
        cu = [int(x) for x in cu_seqlens]
    if cu[0] != 0 or any(b < a for a, b in zip(cu, cu[1:])) or cu[-1] != total:
        raise ValueError("cu_seqlens must start at 0, be non-decreasing and end at the token count")
    return tuple(b - a for a, b in zip(cu, cu[1:]))


def kernel_fn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    state: torch.Tensor | None,
    scale: float | None = None,
    *,
    cu_seqlens=None,
    mode: str = "auto",
    qk_l2norm: bool = False,
    checkpoints: bool = False,
    gates=None,
    segment_chunks: int | None = None,
) -> list[torch.Tensor]:
    nseq, hk, hv = _validate(q, k, v, g, beta, state, cu_seqlens)
    if scale is None:
        scale = D ** -0.5
    dev = q.device
    io_dtype = q.dtype
    B, T = q.shape[0], q.shape[1]
    total = B * T
    if cu_seqlens is None and T == 1 and B > 0 and _mode(mode) == "auto":
        from . import qwen35moe_gdn_decode

        if gates is not None:
            g, beta = gdn_gates(g, beta, *gates)
        res = qwen35moe_gdn_decode.kernel_fn(q, k, v, g, beta, state, scale, qk_l2norm=qk_l2norm)
        return res + [res[1].unsqueeze(1).clone()] if checkpoints else res
    # stage 1 inside the kernels: the gates from the raw projections, and the q/k normalisation
    # of bf16 inputs (fp32 inputs are normalised by the separate pass, which also converts them)
    norm_inside = qk_l2norm and q.dtype == torch.bfloat16
    gate_in, gate_keep = None, ()
    if gates is not None:
        gate_in, gate_keep = _gate_inputs(g, beta, gates, hv)
    if norm_inside:
        gate_in = gate_in if gate_in is not None else _lib.Stage1Inputs()
        gate_in.qk_l2norm = 1
        gate_in.l2norm_eps = QK_L2NORM_EPS
    if cu_seqlens is None:
        lengths = (T,) * B
    else:
        lengths = _lengths(cu_seqlens, T)
    if total == 0:
        out = torch.empty(v.shape, dtype=io_dtype, device=dev)
        fs = state.to(torch.float32).clone() if state is not None else torch.zeros((nseq, hv, D, D), device=dev)
        if checkpoints:
            ck = torch.empty((0, hv, D, D), dtype=torch.float32, device=dev)
            return [out, fs, ck if cu_seqlens is not None else ck.reshape(B, 0, hv, D, D)]
        return [out, fs]
    cu_t, order_t, cb_t, total_chunks, cb_host = _device_meta(lengths, dev)
    qb = l2norm_rows(q) if qk_l2norm and not norm_inside else q.to(torch.bfloat16).contiguous()
    kb = l2norm_rows(k) if qk_l2norm and not norm_inside else k.to(torch.bfloat16).contiguous()
    vb = v.to(torch.bfloat16).contiguous()
    gf = g.to(torch.float32).contiguous() if gates is None else None
    bf = beta.to(torch.float32).contiguous() if gates is None else None
    st = state.to(torch.float32).contiguous() if state is not None else None
    out = torch.empty(vb.shape, dtype=torch.bfloat16, device=dev)
    final_state = torch.empty((nseq, hv, D, D), dtype=torch.float32, device=dev)
    lib = _lib.load()
    word = _lib.status_word(dev)
    gate_ref = ctypes.byref(gate_in) if gate_in is not None else None
    sched, seg_len = _plan(mode, lengths, hv, dev, checkpoints)
    if sched == "segmented" and segment_chunks is not None:
        if int(segment_chunks) < 1:
            raise ValueError("segment_chunks must be positive")
        seg_len = int(segment_chunks)
    ck = torch.empty((total_chunks, hv, D, D), dtype=torch.float32, device=dev) if checkpoints else None
    k_normed = None
    if norm_inside and sched != "fused":  # the preparation writes the normalised keys for the chains
        k_normed = torch.empty_like(kb)
        gate_in.k_normed = k_normed.data_ptr()
    with torch.cuda.device(dev):
        if sched == "segmented":
            cu_host = _host_offsets(lengths)
            nbytes = int(lib.tokmix_gdn_segmented_workspace_bytes(cu_host, nseq, hv, seg_len))
            if nbytes < 0:
                raise ValueError("qwen35moe_gdn_prefill: no segmented plan for these lengths")
            ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
            plan_t = _segment_plan(lengths, cu_host, hv, seg_len, dev)
            rc = lib.tokmix_gdn_prefill_segmented(
                qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), _ptr(gf), _ptr(bf),
                st.data_ptr() if st is not None else None, out.data_ptr(), final_state.data_ptr(),
                cu_t.data_ptr(), cb_t.data_ptr(), cu_host, nseq, total, total_chunks, hk, hv, D, D, float(scale),
                _lib.DTYPE_BF16, gate_ref, seg_len, plan_t.data_ptr(), ws.data_ptr(), ws.numel(), word.data_ptr(),
                _lib.stream_ptr(dev))
        elif sched != "fused":
            nbytes = int(lib.tokmix_gdn_split_workspace_bytes(total_chunks, hv))
            ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
            rec_t = _record_order(lengths, cb_host, hv, dev) if sched == "overlap" else None
            rc = lib.tokmix_gdn_prefill_split(
                qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), _ptr(gf), _ptr(bf),
                st.data_ptr() if st is not None else None, out.data_ptr(), final_state.data_ptr(),
                ck.data_ptr() if ck is not None else None, cu_t.data_ptr(), cb_t.data_ptr(), rec_t.data_ptr() if rec_t is not None else None, nseq, total,
                total_chunks, hk, hv, D, D, float(scale), _lib.DTYPE_BF16, gate_ref, ws.data_ptr(), ws.numel(),
                word.data_ptr(), _lib.stream_ptr(dev))
        else:
            rc = lib.tokmix_gdn_prefill(
                qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), _ptr(gf), _ptr(bf),
                st.data_ptr() if st is not None else None, out.data_ptr(), final_state.data_ptr(),
                cu_t.data_ptr(), order_t.data_ptr() if order_t is not None else None,
                nseq, total, hk, hv, D, D, float(scale), _lib.DTYPE_BF16, gate_ref, word.data_ptr(),
                _lib.stream_ptr(dev))
    _lib.check(rc, "qwen35moe_gdn_prefill")
    _lib.after_launch(dev, "qwen35moe_gdn_prefill")
    if io_dtype != torch.bfloat16:
        out = out.to(io_dtype)
    if ck is not None:
        return [out, final_state, ck if cu_seqlens is not None else ck.reshape(B, total_chunks // B, hv, D, D)]
    return [out, final_state]


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _gate_inputs(a: torch.Tensor, b: torch.Tensor, gates, hv: int):
    """The raw gate projections and per-head parameters as the kernels' gate source (and the
    tensors that must stay alive until the launch)."""
    a_log, dt_bias = gates
    if a.shape != b.shape or a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("gates: a and b must be tensors of one shape and dtype (bf16 or fp32)")
    if tuple(a_log.shape) != (hv,) or tuple(dt_bias.shape) != (hv,):
        raise ValueError(f"gates: A_log and dt_bias must have shape [{hv}]")
    a, b = a.contiguous(), b.contiguous()
    al = a_log.to(device=a.device, dtype=torch.float32).contiguous()
    db = dt_bias.to(device=a.device, dtype=torch.float32).contiguous()
    src = _lib.Stage1Inputs(a.data_ptr(), b.data_ptr(), _lib.DTYPE_BF16 if a.dtype == torch.bfloat16 else _lib.DTYPE_FP32,
                          al.data_ptr(), db.data_ptr())
    return src, (a, b, al, db)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    """g = -exp(a_log) * softplus(a + dt_bias), beta = sigmoid(b) on the device in fp32
    (``tokmix_gdn_gates``).  a, b: [..., Hv] bf16 or fp32 CUDA tensors; a_log, dt_bias: [Hv]."""
    if a.shape != b.shape or a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float32) or not a.is_cuda:
        raise ValueError("gates: a and b must be CUDA tensors of one shape and dtype (bf16 or fp32)")
    hv = a.shape[-1]
    if tuple(a_log.shape) != (hv,) or tuple(dt_bias.shape) != (hv,):
        raise ValueError(f"gates: A_log and dt_bias must have shape [{hv}]")
    a, b = a.contiguous(), b.contiguous()
    al = a_log.to(device=a.device, dtype=torch.float32).contiguous()
    db = dt_bias.to(device=a.device, dtype=torch.float32).contiguous()
    g = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    beta = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        rc = _lib.load().tokmix_gdn_gates(
            a.data_ptr(), b.data_ptr(), _lib.DTYPE_BF16 if a.dtype == torch.bfloat16 else _lib.DTYPE_FP32, al.data_ptr(),
            db.data_ptr(), g.data_ptr(), beta.data_ptr(), a.numel() // hv, hv, _lib.stream_ptr(a.device))
    _lib.check(rc, "gdn_gates")
    return g, beta


def l2norm_rows(x: torch.Tensor, eps: float = QK_L2NORM_EPS) -> torch.Tensor:
    """x / sqrt(sum(x^2, last dim) + eps) per 128-element row, fp32 arithmetic, bf16 result
    (``tokmix_l2norm_rows``).  x: bf16 or fp32 CUDA tensor whose last dimension is 128."""
    if x.shape[-1] != D or x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda:
        raise ValueError("l2norm_rows takes a bf16 or fp32 CUDA tensor with last dimension 128")
    x = x.contiguous()
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    rows = x.numel() // D
    with torch.cuda.device(x.device):
        rc = _lib.load().tokmix_l2norm_rows(
            x.data_ptr(), _lib.DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.DTYPE_FP32, y.data_ptr(), rows, D,
            float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "l2norm_rows")
    return y


def _record_order(lengths: tuple[int, ...], chunk_base: list[int], hv: int, device: torch.device) -> torch.Tensor:
    """Records (global chunk * hv + value head) in chunk-major order: the order in which the
    overlapped split launch prepares them, so that every chain's next chunk is ready first."""
    key = ("order", lengths, hv, device)
    hit = _meta_cache.get(key)
    if hit is None:
        nch = [(n + 63) // 64 for n in lengths]
        rec = [(chunk_base[s] + c) * hv + h for c in range(max(nch, default=0))
               for s in range(len(lengths)) if c < nch[s] for h in range(hv)]
        hit = torch.tensor(rec if rec else [0], dtype=torch.int32).to(device)
        _meta_cache[key] = hit
    return hit


def _mode(mode: str) -> str:
    if mode == "auto":
        mode = os.environ.get("TOKMIX_GDN_MODE", "auto")
    if mode not in ("auto", "fused", "split", "overlap", "segmented"):
        raise ValueError(f"mode must be 'auto', 'fused', 'split', 'overlap' or 'segmented' (got {mode!r})")
    return mode


def _host_offsets(lengths: tuple[int, ...]):
    """cu_seqlens as a host int32 array for the C ABI (the segment plan is made on the host)."""
    key = ("cu_host", lengths)
    hit = _meta_cache.get(key)
    if hit is None:
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + n)
        hit = (ctypes.c_int32 * len(cu))(*cu)
        _meta_cache[key] = hit
    return hit


def _segment_plan(lengths: tuple[int, ...], cu_host, hv: int, seg_len: int, device: torch.device) -> torch.Tensor:
    """The segmented schedule's tables (``tokmix_gdn_segmented_plan``) on the device, made and
    uploaded once per shape, so that a call enqueues no host-to-device copy."""
    key = ("segplan", lengths, hv, seg_len, device)
    hit = _meta_cache.get(key)
    if hit is None:
        lib = _lib.load()
        nbytes = int(lib.tokmix_gdn_segmented_plan_bytes(cu_host, len(lengths), hv, seg_len))
        if nbytes < 0:
            raise ValueError("qwen35moe_gdn_prefill: no segmented plan for these lengths")
        host = torch.zeros(max(nbytes, 16), dtype=torch.uint8)
        _lib.check(lib.tokmix_gdn_segmented_plan(cu_host, len(lengths), hv, seg_len, host.data_ptr(), host.numel()),
                   "tokmix_gdn_segmented_plan")
        hit = host.to(device)
        _meta_cache[key] = hit
    return hit


def _segment_units(nchunks: list[int], seg_len: int) -> tuple[int, int, int]:
    """(chain units per head, most segments of one sequence, chunks in later segments) when
    sequences longer than seg_len chunks are cut into the fewest near-equal segments of at most
    seg_len chunks: a whole sequence is one chain, a cut one 2 s - 1 (its first segment, then
    each later segment twice)."""
    units, most, later = 0, 1, 0
    for n in nchunks:
        s = -(-n // seg_len) if n > seg_len else 1
        units += 2 * s - 1
        most = max(most, s)
        if s > 1:
            later += n - (n // s + (1 if n % s else 0))
    return units, most, later


def segment_length(lengths, hv: int, sms: int) -> int | None:
    """The segment length (chunks) of the segmented schedule: the shortest whose chains
    (units x hv) still fit on the SMs at once, no shorter than _SEG_MIN_CHUNKS; None when cutting
    gains nothing (no sequence longer than that length)."""
    nch = [(n + 63) // 64 for n in lengths]
    longest = max(nch, default=0)
    best = None
    for seg in range(longest - 1, _SEG_MIN_CHUNKS - 1, -1):
        units = _segment_units(nch, seg)[0]
        if units * hv > sms:
            break
        best = seg
    return best


def _predicted_us(sched: str, units: int, records: int, max_chunks: int, sms: int, segs: int = 1,
                  later_chunks: int = 0, hv: int = 0) -> float:
    """Predicted time of one schedule for `units` chains (all on the SMs at once) whose longest
    has `max_chunks` chunks, with `records` preparation records in all (for "segmented": the
    longest segment, `segs` segments in the most-cut sequence and `later_chunks` chunks in later
    segments, per value head of the hv)."""
    if sched == "fused":
        return max_chunks * _US_FUSED_CHUNK
    if sched == "overlap":  # the chains and 3 preparation groups on each remaining SM
        prep = records * _US_PREP_RECORD_OVERLAP / (3 * (sms - units))
        return max(max_chunks * _US_CHAIN_CHUNK, prep) + _US_OVERLAP_START
    prep = records * _US_PREP_RECORD / (3 * sms)
    if sched == "segmented":
        corr = later_chunks * 64 * hv * 768 / _SEG_CORR_BYTES_PER_US
        return (prep + _US_SEG_CHAIN_START + max_chunks * _US_SEG_CHAIN_CHUNK + _US_SEG_COMBINE_START
                + (segs - 1) * _US_SEG_COMBINE_STEP + _US_SEG_CORR_START + corr + _US_SEG_GAPS)
    return prep + max_chunks * _US_CHAIN_CHUNK + _US_SPLIT_GAP


def _plan(mode: str, lengths: tuple[int, ...], hv: int, dev: torch.device,
          checkpoints: bool = False) -> tuple[str, int]:
    """_plan_uncached, memoised per shape (the search over segment lengths is host work that a
    repeated call should not pay again)."""
    key = ("plan", _mode(mode), lengths, hv, dev, checkpoints)
    hit = _meta_cache.get(key)
    if hit is None:
        hit = _plan_uncached(mode, lengths, hv, dev, checkpoints)
        _meta_cache[key] = hit
    return hit


def _plan_uncached(mode: str, lengths: tuple[int, ...], hv: int, dev: torch.device,
                   checkpoints: bool = False) -> tuple[str, int]:
    """(schedule, segment length in chunks -- 0 unless "segmented").  "auto": "fused" when one
    CTA per unit fills the SMs (or the workspace would be too large); otherwise the schedule with
    the lowest predicted time (`_predicted_us`) among "fused", "overlap" (possible when the
    chains leave at least 8 SMs to the preparation CTAs), "split" and "segmented" (possible when
    some sequence is long enough to cut).  With checkpoints only "split" and "overlap" qualify."""
    mode = _mode(mode)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    units = len(lengths) * hv
    nch = [(n + 63) // 64 for n in lengths]
    total_chunks, max_chunks = sum(nch), max(nch, default=0)
    seg = segment_length(lengths, hv, sms) if not checkpoints else None
    if mode != "auto":
        if checkpoints and mode in ("fused", "segmented"):
            raise ValueError(f"checkpoints need the split or overlap schedule (mode={mode!r} given)")
        if mode == "segmented":
            return mode, seg if seg is not None else max(max_chunks, 1)
        return mode, 0
    too_big = _lib.load().tokmix_gdn_split_workspace_bytes(total_chunks, hv) > _SPLIT_MAX_WORKSPACE
    if units >= sms:
        # several waves of units: the one-CTA-per-unit kernel (longest first), or every record
        # prepared first and the chains run longest first (the segmented launch without cuts)
        if checkpoints:
            return "split", 0
        if too_big:
            return "fused", 0
        work = total_chunks * hv
        fused = max(max_chunks * _US_FUSED_CHUNK, work * _US_FUSED_CHUNK_WAVES / sms)
        lpt = (total_chunks * hv * _US_PREP_RECORD / (3 * sms) + _US_SPLIT_GAP +
               max(max_chunks, work / sms) * _US_SEG_CHAIN_CHUNK)
        return ("segmented", max(max_chunks, 1)) if lpt < fused else ("fused", 0)
    if not checkpoints and too_big:
        return "fused", 0
    records = total_chunks * hv
    # ties go to the earlier entry: the single fused launch first
    cands = ([] if checkpoints else ["fused"]) + (["overlap"] if units + 8 <= sms else []) + ["split"]
    pred = {c: _predicted_us(c, units, records, max_chunks, sms) for c in cands}
    if seg is not None:
        seg_units, most, later = _segment_units(nch, seg)
        pred["segmented"] = _predicted_us("segmented", seg_units * hv, records, seg, sms, most, later, hv)
    best = min(pred, key=pred.get)
    return best, seg if best == "segmented" else 0


def _schedule(mode: str, units: int, total_chunks: int, hv: int, dev: torch.device,
              checkpoints: bool = False, max_chunks: int | None = None) -> str:
    """The schedule for `units` / hv sequences of equal chunk counts (see _plan)."""
    n = max(1, units // hv)
    per = max_chunks if max_chunks is not None else -(-total_chunks // n)
    return _plan(mode, (per * 64,) * n, hv, dev, checkpoints)[0]


def schedule(q: torch.Tensor, v: torch.Tensor, cu_seqlens=None, mode: str = "auto") -> str:
    """The schedule kernel_fn picks for these inputs: "fused", "split", "overlap", "segmented"
    or "decode"."""
    B, T, hv = q.shape[0], q.shape[1], v.shape[2]
    if cu_seqlens is None and T == 1 and B > 0 and _mode(mode) == "auto":
        return "decode"
    lengths = (T,) * B if cu_seqlens is None else _lengths(cu_seqlens, T)
    return _plan(mode, lengths, hv, q.device)[0]


def check_device_status(device: torch.device | None = None) -> None:
    """Synchronise and raise if any kernel on `device` reported a device-side timeout."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    _lib.check_status(dev, "qwen35moe_gdn_prefill")


def filled(shape, scale: float, bias: float, dtype=torch.float32, device="cuda") -> torch.Tensor:
    """The reference's deterministic fixture ``((i mod 251) - 125) * scale + bias``
    (``kernels/qwen35moe_gdn_prefill.py:158-164``)."""
    n = 1
    for dim in shape:
        n *= dim
    x = torch.arange(n, device=device, dtype=torch.float32)
    x = ((x % 251) - 125.0) * scale + bias
    return x.reshape(shape).to(dtype)


def get_inputs(batch: int = 1, seq_len: int = 4096, dtype: torch.dtype = torch.float32, seed: int = 42,
               device: str = "cuda") -> dict:
    """The reference's fixture (``kernels/qwen35moe_gdn_prefill.py:154-174``; seed ignored)."""
    del seed
    return {
        "q": filled((batch, seq_len, H_K, D), 0.001, 0.0, dtype, device),
        "k": filled((batch, seq_len, H_K, D), 0.001, 0.0, dtype, device),
        "v": filled((batch, seq_len, H_V, D), 0.001, 0.0, dtype, device),
        "g": filled((batch, seq_len, H_V), 0.0001, -0.01, torch.float32, device),
        "beta": filled((batch, seq_len, H_V), 0.0001, 0.5, torch.float32, device),
        "state": filled((batch, H_V, D, D), 0.0001, 0.0, torch.float32, device),
        "scale": D ** -0.5,
    }


def get_flops(batch: int = 1, seq_len: int = 4096) -> int:
    """Reference formula (recurrent count), ``kernels_optimized/qwen35moe_gdn_prefill.py:170-171``."""
    return 4 * batch * H_V * seq_len * D * D


def get_bytes(batch: int = 1, seq_len: int = 4096, element_size: int = 4) -> int:
    """Reference formula, ``kernels_optimized/qwen35moe_gdn_prefill.py:174-179`` (one element
    size for every tensor)."""
    qk = 2 * batch * seq_len * H_K * D
    vo = 2 * batch * seq_len * H_V * D
    gb = 2 * batch * seq_len * H_V
    st = 2 * batch * H_V * D * D
    return (qk + vo + gb + st) * element_size


def algorithmic_bytes(tokens: int, n_seqs: int, hk: int = H_K, hv: int = H_V, io_bytes: int = 2) -> int:
    """Bytes the bf16-I/O kernel must move at minimum: q, k, v read and o written in `io_bytes`
    per element, g and beta read in fp32, one fp32 state read and written per (sequence, head)."""
    return (tokens * (2 * hk + 2 * hv) * D * io_bytes + tokens * 2 * hv * 4 + n_seqs * hv * D * D * 4 * 2)
