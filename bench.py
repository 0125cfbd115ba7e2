"""Benchmark of the B200 prefill token mixers (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workloads (synthetic data from fixed seeds, shapes of the B200 configs):
  gdn_b1_t2048   (default, headline)  GDN prefill B=1 T=2048 Hk=16 Hv=32 d=128, chunk 64, bf16 q/k/v/o,
                 fp32 g/beta/state, zero initial state.  Weak scaling: every rank runs its own batch.
  gdn_b1_t2048_heads  the same single batch strong-scaled: the 16 key heads (with the value heads
                 reading them) split across the ranks (at N > 1 under "also").
  fa2_b4_s8192   FA2 causal GQA forward B=4 Hq=32 Hkv=8 S=8192 D=128 bf16.  Strong scaling: the
                 8 key/value heads (with their 4 query heads each) are split across ranks.  Carries
                 its own end-to-end leg, the CPU oracle on a sample, and torch SDPA (the reference's
                 FA2 oracle) timed on the same inputs as a same-box comparator.
  gdn_varlen     GDN prefill, 8 sequences of U[1024, 32768] tokens packed with cu_seqlens,
                 per-sequence initial state N(0, 0.02).  Strong scaling over head groups.
  gdn_decode_b128  one GDN decode token for 128 sequences, states updated in place.
  hybrid_t4096 / hybrid_t16384 / hybrid_t65536  (opt-in with --workload; minutes at T=65536)
                 the hybrid prefill sweep: FA2 causal GQA Hq=16 Hkv=2 D=256 plus GDN prefill Hk=16
                 Hv=32 d=128, both at B=16 and sequence length T, the batch split across the ranks.
The headline line also carries the other workloads under "also" (same run, same timing rules), and
on one GPU the three row-wise plugin ops (rms_norm M=16384 N=5120 bf16; swiglu_input_quant
M=4096 N=7168; qkv_part_rope B=50 S=2048 12 heads of 256, nope 192) in GB/s of the bytes their
configs count, and FA2 head_dim 256 (fa2_d256_b16_s4096: causal GQA B=16 Hq=16 Hkv=2 S=4096).

Timing: W untimed warm-up steps, then K timed steps bracketed by a barrier and
torch.cuda.synchronize(); each step is timed with CUDA events on the launching stream and the
L2 cache (126 MB) is flushed by writing a 256 MB buffer between steps when the step's inputs fit
in L2.  The step time is the max over ranks.  `e2e` repeats the headline step through the public
plugin call from pinned host buffers, host->device copies of the inputs and device->host copies
of the outputs inside the timed region, as a serving loop runs them: each step's uploads overlap
the previous step's kernel and read-back (two copy streams, two input buffers).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from kernel_opt_agent_b200 import flash_attention_2 as fa2  # noqa: E402
from kernel_opt_agent_b200 import qwen35moe_gdn_decode as gdn_dec  # noqa: E402
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn  # noqa: E402
from kernel_opt_agent_b200 import qkv_part_rope as rope_op  # noqa: E402
from kernel_opt_agent_b200 import rms_norm as rms_op  # noqa: E402
from kernel_opt_agent_b200 import sharding  # noqa: E402
from kernel_opt_agent_b200 import swiglu_input_quant as swiglu_op  # noqa: E402
from kernel_opt_agent_b200.kernel_configs import KERNEL_CONFIGS  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
D = 128
HK, HV = 16, 32
# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of each workload's
# kernel(s) from one ncu capture, keyed "workload/schedule".  ncu replays each kernel with flushed
# caches, so for the split GDN schedule the chain kernel's reads of the records (which stay in L2
# in a real run) count as DRAM reads.  FA2: captured at batch 1 (the batch-4 inputs exceed the
# capture size rule) and scaled by 4.
NCU_TRAFFIC_BYTES = {
    "gdn_b1_t2048/overlap": 45_328_640 + 49_478_656,
    "gdn_b1_t2048/split": 17_699_072 + 23_969_536 + 104_127_488 + 7_339_264,  # prep + chain
    "gdn_b1_t2048/fused": 36_302_848 + 54_016,
    "fa2_b4_s8192/fused": 4 * (101_431_808 + 32_353_792),
    "gdn_decode_b128/decode": 270_583_808 + 210_555_648,
    "rms_norm_m16384_n5120/row_op": 167_820_032 + 111_249_664,
    "swiglu_quant_m4096_n7168/row_op": 117_454_848 + 69_972_480,
    "qkv_rope_b50_s2048/row_op": 629_694_464 + 579_417_344,
    # FA2 head_dim 256: captured at batch 4 (the batch-16 inputs exceed the capture size rule), x4
    "fa2_d256_b16_s4096/fused": 4 * (169_233_152 + 92_687_872),
    "fa2_d256_b4_s4096/fused": 169_233_152 + 92_687_872,
}


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ----------------------------------------------------------------------------- input generation
def gdn_inputs(device, tokens_per_seq, seed, lengths=None, state_std=0.0, hk=HK, hv=HV):
    """GDN workload drawn on the device from a seeded generator (q, k L2-normalised, v ~ N(0,1),
    g = -softplus(N(0,1)), beta = sigmoid(N(0,1)))."""
    gen = torch.Generator(device=device).manual_seed(seed)
    T = int(sum(lengths)) if lengths is not None else tokens_per_seq
    nseq = len(lengths) if lengths is not None else 1
    q = torch.randn(1, T, hk, D, device=device, generator=gen)
    k = torch.randn(1, T, hk, D, device=device, generator=gen)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(1, T, hv, D, device=device, generator=gen).to(torch.bfloat16)
    g = -torch.nn.functional.softplus(torch.randn(1, T, hv, device=device, generator=gen))
    beta = torch.sigmoid(torch.randn(1, T, hv, device=device, generator=gen))
    state = torch.randn(nseq, hv, D, D, device=device, generator=gen) * state_std
    inp = {"q": q, "k": k, "v": v, "g": g, "beta": beta, "state": state, "scale": D ** -0.5}
    if lengths is not None:
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + int(n))
        inp["cu_seqlens"] = torch.tensor(cu, dtype=torch.int32)
    return inp


def varlen_lengths(n=8, lo=1024, hi=32768, seed=0):
    gen = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=gen)]


def fa2_inputs(device, batch, hq, hkv, s, d, seed):
    """q, k, v ~ N(0,1) drawn on the device from a seeded generator (same values on every rank)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(batch, hq, s, d, device=device, generator=gen, dtype=torch.bfloat16)
    k = torch.randn(batch, hkv, s, d, device=device, generator=gen, dtype=torch.bfloat16)
    v = torch.randn(batch, hkv, s, d, device=device, generator=gen, dtype=torch.bfloat16)
    return {"q": q, "k": k, "v": v, "causal": True, "sm_scale": 1.0 / math.sqrt(d)}


def input_bytes(inp) -> int:
    return sum(t.numel() * t.element_size() for t in inp.values() if isinstance(t, torch.Tensor) and t.is_cuda)


# ----------------------------------------------------------------------------- timing helpers
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while GPU work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", ",".join(str(g) for g in gpus)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons, n = [], [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            n += 1
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": n}


def max_over_ranks(x: float, device) -> float:
    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def time_steps(step_fn, steps, warmup, device, flush: bool, collective: bool = True):
    """Runs warmup + steps; returns (max-over-ranks total seconds of the K timed steps, per-step ms
    list).  collective=False: this rank alone (no barrier, no max over ranks)."""
    flush_buf = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device) if flush else None
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        if flush_buf is not None:
            flush_buf.fill_(1)
        step_fn()
    torch.cuda.synchronize(device)
    if collective:
        barrier()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        if flush_buf is not None:
            flush_buf.fill_(i & 0xFF)
        starts[i].record(stream)
        step_fn()
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    if collective:
        barrier()
    torch.cuda.synchronize(device)
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_s = sum(per) / 1e3
    return (max_over_ranks(total_s, device) if collective else total_s), per


def stage_arenas(tensors, device):
    """A step's inputs staged in one pinned host buffer (filled with `tensors`' values) and two
    device buffers of the same layout, so that a step uploads them with one copy; returns (host
    buffer, [device buffers], views) where views(buffer) gives the tensors as views of a buffer
    (256-byte aligned)."""
    offsets, total = {}, 0
    for k, v in tensors.items():
        offsets[k] = total
        total += -(-v.numel() * v.element_size() // 256) * 256

    def views(arena):
        return {k: arena[offsets[k]:offsets[k] + v.numel() * v.element_size()].view(v.dtype).view(v.shape)
                for k, v in tensors.items()}

    host_arena = torch.empty(total, dtype=torch.uint8).pin_memory()
    for k, v in views(host_arena).items():
        v.copy_(tensors[k].cpu())
    return host_arena, [torch.empty(total, dtype=torch.uint8, device=device) for _ in range(2)], views


PIPELINE_NOTE = ("each step uploads its inputs (staged in one pinned buffer: one copy) and reads back its "
                 "results; step i+1's upload runs beside step i's kernel and read-back (two copy streams, two "
                 "input buffers)")


def time_pipelined(upload, compute, download, steps, warmup, device, collective: bool = True):
    """End-to-end steps as a serving loop runs them: step i's uploads (host -> device, on one copy
    stream, into input buffer i % 2) run beside step i-1's kernel and step i-2's read-back (device ->
    host, on a second copy stream), ordered by events; every step still uploads its own inputs and
    reads back its own results.  upload(b) and download(b, outs) issue copies on the current stream
    (set to the copy stream by the caller), compute(b) runs the kernel on the device's current
    stream and returns the output tensors.  Returns the max-over-ranks seconds of the K timed steps:
    from an event the first upload waits on to the end of the last read-back."""
    s_c = torch.cuda.current_stream(device)
    s_up, s_dn = torch.cuda.Stream(device), torch.cuda.Stream(device)
    comp_done = [None, None]

    def run(n, first_wait=None):
        last = None
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(s_up):
                if i == 0 and first_wait is not None:
                    s_up.wait_event(first_wait)
                if comp_done[b] is not None:  # the kernel that last read buffer b is done
                    s_up.wait_event(comp_done[b])
                upload(b)
            up = torch.cuda.Event()
            up.record(s_up)
            s_c.wait_event(up)
            outs = compute(b)
            done = torch.cuda.Event()
            done.record(s_c)
            comp_done[b] = done
            s_dn.wait_event(done)
            with torch.cuda.stream(s_dn):
                for t in outs:
                    t.record_stream(s_dn)
                download(b, outs)
            last = torch.cuda.Event(enable_timing=True)
            last.record(s_dn)
        return last

    run(warmup)
    torch.cuda.synchronize(device)
    if collective:
        barrier()
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    start.record(s_c)
    end_dn = run(steps, first_wait=start)
    s_c.wait_event(end_dn)
    end = torch.cuda.Event(enable_timing=True)
    end.record(s_c)
    torch.cuda.synchronize(device)
    if collective:
        barrier()
    torch.cuda.synchronize(device)
    total_s = start.elapsed_time(end) / 1e3
    return max_over_ranks(total_s, device) if collective else total_s


# ----------------------------------------------------------------------------- workloads
def run_gdn_batch(device, rank, world, steps, warmup, batch=1):
    inp = gdn_inputs(device, 2048, seed=1000 + rank, lengths=[2048] * batch if batch > 1 else None)
    tokens = 2048 * batch * world
    total_s, per = time_steps(lambda: gdn.kernel_fn(**inp), steps, warmup, device,
                              flush=input_bytes(inp) < L2_BYTES)
    gdn.check_device_status(device)
    algo = gdn.algorithmic_bytes(2048 * batch, batch)
    ms = total_s / steps * 1e3
    return {"tokens_per_step": tokens, "ms": ms, "value": tokens * steps / total_s / 1e6, "unit": "Mtok/s",
            "kernel_ms_local": statistics.mean(per), "algo_bytes": algo, "inp": inp,
            "token_heads": 2048 * batch * HV, "schedule": gdn.schedule(inp["q"], inp["v"])}


def headline_config(world: int) -> dict:
    return {"workload": "gdn_b1_t2048", "batch_per_rank": 1, "seq_len": 2048, "hk": HK, "hv": HV, "head_dim": D,
            "chunk": 64, "io": "bf16 q/k/v/o, fp32 g/beta/state", "initial_state": "zero",
            "parallelism": f"dp{world} (one batch per rank)", "l2": "flushed between timed steps (256 MB write)"}


HEADLINE_METRIC = "GDN prefill Mtok/s"
SPEC_HBM_GBS = 8000.0       # nominal HBM3e bandwidth, for context beside the measured copy peak
SPEC_BF16_TFLOPS = 2250.0   # nominal dense bf16 tensor throughput
# tensor-core work of the chunked GDN form per token and value head (C = 64, D = 128):
# 6 D^2 for the state products plus 8 C D for the in-chunk products
GDN_CHUNKED_FLOP_PER_TOKEN_HEAD = 6 * 128 * 128 + 8 * 64 * 128


def run_gdn_varlen(device, rank, world, steps, warmup, verify=False):
    lengths = varlen_lengths()
    full = gdn_inputs(device, 0, seed=7, lengths=lengths, state_std=0.02)
    ranges = sharding.even_ranges(HK, world)
    a, b = ranges[rank]
    inp = sharding.slice_gdn_inputs(full, a, b)
    if not verify:
        del full
    tokens = sum(lengths)
    total_s, per = time_steps(lambda: gdn.kernel_fn(**inp), steps, warmup, device,
                              flush=input_bytes(inp) < L2_BYTES)
    gdn.check_device_status(device)
    algo = gdn.algorithmic_bytes(tokens, len(lengths), hk=b - a, hv=2 * (b - a))
    res = {"tokens_per_step": tokens, "ms": total_s / steps * 1e3, "value": tokens * steps / total_s / 1e6,
           "unit": "Mtok/s", "kernel_ms_local": statistics.mean(per), "algo_bytes": algo,
           "token_heads": tokens * 2 * (b - a), "schedule": gdn.schedule(inp["q"], inp["v"], inp.get("cu_seqlens")),
           "config": {"workload": "gdn_varlen", "n_seqs": 8, "lengths": lengths, "total_tokens": tokens,
                      "hk": HK, "hv": HV, "head_dim": D, "chunk": 64, "initial_state": "N(0,0.02)",
                      "shard": f"key heads {HK // world}/rank (+ the value heads reading them); the rank's "
                               "schedule cuts long sequences into segments chained side by side when that is "
                               "predicted faster"}}
    if verify and world > 1:
        out, fs = gdn.kernel_fn(**inp)
        go = sharding.gather_to_rank0(out, dim=2)
        gs = sharding.gather_to_rank0(fs, dim=1)
        if rank == 0:
            ref_o, ref_s = gdn.kernel_fn(**full)
            sizes = [2 * (y - x) for x, y in ranges]
            offs = [sum(sizes[:i]) for i in range(world)]
            o = sharding.unscatter_gdn_heads([go.narrow(2, o0, n) for o0, n in zip(offs, sizes)], ranges, HK, HV, 2)
            st = sharding.unscatter_gdn_heads([gs.narrow(1, o0, n) for o0, n in zip(offs, sizes)], ranges, HK, HV, 1)
            res.update(compare_gdn(o, st, ref_o, ref_s))
    return res


def compare_gdn(o, st, ref_o, ref_s) -> dict:
    """Gathered GDN outputs against a one-GPU run: bit for bit when both ran schedules that issue
    the same operations (fused / split / overlap), else within the parity tests' tolerances (the
    segmented schedule rounds its later segments' outputs once more)."""
    bitwise = bool(torch.equal(o, ref_o) and torch.equal(st, ref_s))
    close = bool(torch.allclose(o.float(), ref_o.float(), atol=2e-2, rtol=2e-2) and
                 torch.allclose(st, ref_s, atol=1e-4, rtol=1e-3))
    return {"verified_vs_one_gpu": bitwise or close, "bitwise_vs_one_gpu": bitwise,
            "max_abs_diff_vs_one_gpu": {"out": float((o.float() - ref_o.float()).abs().max()),
                                        "state": float((st - ref_s).abs().max())}}


def run_gdn_decode(device, rank, world, steps, warmup, batch=128):
    """One decode token for each of `batch` sequences (split over the ranks), Hk16 Hv32, states
    N(0, 0.02) updated in place every step as in a decode loop.  L2 is flushed between steps: a
    rank's share of the 268 MB of state is close to or below the L2 size at 2 or more GPUs."""
    local = batch // world
    inp = gdn_dec.get_inputs(batch=local, seed=5000 + rank, device=str(device))
    total_s, per = time_steps(lambda: gdn_dec.kernel_fn(**inp, inplace=True), steps, warmup, device, flush=True)
    algo = gdn_dec.algorithmic_bytes(local)
    return {"tokens_per_step": batch, "ms": total_s / steps * 1e3, "value": batch * steps / total_s / 1e6,
            "unit": "Mtok/s", "kernel_ms_local": statistics.mean(per), "algo_bytes": algo, "schedule": "decode",
            "config": {"workload": "gdn_decode_b128", "batch": batch, "tokens_per_sequence": 1, "hk": HK, "hv": HV,
                       "head_dim": D, "state": "N(0,0.02) fp32, updated in place",
                       "l2": "flushed between timed steps (256 MB write)", "shard": f"sequences {local}/rank"}}


# the row-wise plugin ops: (module, config name, size, dtype, kernel symbol)
ROW_OPS = {
    "rms_norm_m16384_n5120": (rms_op, "rms_norm", {"M": 16384, "N": 5120}, torch.bfloat16,
                              "tokmix::ops::rms_norm_kernel<__nv_bfloat16>"),
    "swiglu_quant_m4096_n7168": (swiglu_op, "swiglu_input_quant", {"M": 4096, "N": 7168}, torch.bfloat16,
                                 "tokmix::ops::swiglu_quant_kernel"),
    "qkv_rope_b50_s2048": (rope_op, "qkv_part_rope", {"batch": 50, "seq_len": 2048, "q_heads": 10, "kv_heads": 1,
                                                      "head_dim": 256, "nope_dim": 192}, torch.bfloat16,
                           "tokmix::ops::qkv_part_rope_kernel"),
}


def run_row_op(device, steps, warmup, name):
    """One call of a row-wise plugin op on its config's inputs; value = the config's byte count
    (bytes_fn) per second.  L2 is flushed between steps."""
    mod, cname, size, dtype, kern = ROW_OPS[name]
    cfg = KERNEL_CONFIGS[cname]
    inp = cfg["input_generator"](size, dtype, str(device), seed=7)
    total_s, per = time_steps(lambda: mod.kernel_fn(**inp), steps, warmup, device, flush=True)
    algo = cfg["bytes_fn"](size, dtype)
    ms = total_s / steps * 1e3
    return {"ms": ms, "value": algo / (total_s / steps) / 1e9, "unit": "GB/s", "kernel_ms_local": statistics.mean(per),
            "algo_bytes": algo, "schedule": "row_op", "kernel": kern,
            "config": {"workload": name, **size, "dtype": str(dtype).replace("torch.", ""),
                       "l2": "flushed between timed steps (256 MB write)"}}


def run_fa2(device, rank, world, steps, warmup, batch=4, verify=False, extras=False):
    """FA2 causal GQA B4 Hq32 Hkv8 S8192 D128, key/value heads split across the ranks.  With
    `extras`: the end-to-end leg and (one GPU) the torch SDPA comparators."""
    B, HQ, HKV, S, DD = batch, 32, 8, 8192, 128
    ranges = sharding.even_ranges(HKV, world)
    a, b = ranges[rank]
    full = fa2_inputs(device, B, HQ, HKV, S, DD, seed=3)
    inp = sharding.slice_fa2_inputs(full, a, b)
    if not verify:
        del full
    flops_total = fa2.get_flops(B, HQ, S, DD, causal=True)
    total_s, per = time_steps(lambda: fa2.kernel_fn(**inp), steps, warmup, device,
                              flush=input_bytes(inp) < L2_BYTES)
    fa2.check_device_status(device)
    local_flops = fa2.get_flops(B, (b - a) * (HQ // HKV), S, DD, causal=True)
    res = {"ms": total_s / steps * 1e3, "value": flops_total * steps / total_s / 1e12, "unit": "TFLOP/s",
           "kernel_ms_local": statistics.mean(per), "local_flops": local_flops,
           "config": {"workload": f"fa2_b{B}_s8192", "batch": B, "heads_q": HQ, "heads_kv": HKV, "seq_len": S,
                      "head_dim": DD, "causal": True, "layout": "bhsd",
                      "shard": f"kv heads {HKV // world}/rank (+ their query heads)"}}
    if verify and world > 1:
        got = sharding.gather_to_rank0(fa2.kernel_fn(**inp), dim=1)
        if rank == 0:
            res["verified_vs_one_gpu"] = bool(torch.equal(got, fa2.kernel_fn(**full)))
    if extras:
        res["e2e"] = e2e_fa2(device, inp, max(3, steps // 2), warmup, flops_total)
        if world == 1:
            res["sdpa"] = sdpa_comparators(inp, flops_total, steps, warmup, device)
    return res


def run_fa2_d256(device, steps, warmup, batch=16):
    """FA2 head_dim 256, the hybrid configuration's attention: causal GQA B16 Hq16 Hkv2 S4096
    (batch 4: the profiling-size case, inputs above L2), one GPU (the fa2::d256 kernel)."""
    B, HQ, HKV, S, DD = batch, 16, 2, 4096, 256
    inp = fa2_inputs(device, B, HQ, HKV, S, DD, seed=4)
    flops = fa2.get_flops(B, HQ, S, DD, causal=True)
    total_s, per = time_steps(lambda: fa2.kernel_fn(**inp), steps, warmup, device,
                              flush=input_bytes(inp) < L2_BYTES)
    fa2.check_device_status(device)
    return {"ms": total_s / steps * 1e3, "value": flops * steps / total_s / 1e12, "unit": "TFLOP/s",
            "kernel_ms_local": statistics.mean(per), "local_flops": flops,
            "kernel": "tokmix::fa2::d256::fa2_fwd_d256_kernel",
            "sdpa": sdpa_comparators(inp, flops, steps, warmup, device),
            "config": {"workload": f"fa2_d256_b{B}_s4096", "batch": B, "heads_q": HQ, "heads_kv": HKV, "seq_len": S,
                       "head_dim": DD, "causal": True, "layout": "bhsd"}}


def sdpa_comparators(inp, flops, steps, warmup, device):
    """torch.nn.functional.scaled_dot_product_attention -- the reference's FA2 oracle and comparator
    (``references/flash_attention_2.py:33-41``, paired with ``kernel_fn`` in ``tools/bench.py``) --
    on the same device inputs with the same timing, once per backend that accepts the shape
    (NVIDIA's own attention kernels for this GPU are among them).  TFLOP/s of the same flop count."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    q, k, v = inp["q"], inp["k"], inp["v"]
    gqa = q.shape[1] != k.shape[1]
    res = {}
    for name, backend in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION),
                          ("efficient", SDPBackend.EFFICIENT_ATTENTION)):
        def call():
            with sdpa_kernel(backend):
                return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True,
                                                                        scale=inp["sm_scale"], enable_gqa=gqa)
        try:
            call()
            torch.cuda.synchronize(device)
        except RuntimeError as e:  # backend does not take this shape / GPU
            res[name] = {"unavailable": str(e).splitlines()[0][:160]}
            continue
        total_s, _ = time_steps(call, steps, warmup, device, flush=input_bytes(inp) < L2_BYTES, collective=False)
        res[name] = {"value": flops * steps / total_s / 1e12, "unit": "TFLOP/s", "ms": total_s / steps * 1e3}
    return res


def e2e_fa2(device, inp, steps, warmup, flops_total):
    """FA2 step through the public plugin call from pinned host memory: every step uploads q, k, v,
    runs kernel_fn and reads back the output, pipelined as a serving loop runs it (time_pipelined)."""
    tensors = {n: inp[n] for n in ("q", "k", "v")}
    host_arena, dev_arena, views = stage_arenas(tensors, device)
    dev_bufs = [views(a) for a in dev_arena]
    out_host = [torch.empty(tensors["q"].shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in tensors.values())
    d2h = out_host[0].numel() * 2

    def upload(b):
        dev_arena[b].copy_(host_arena, non_blocking=True)

    def compute(b):
        d = dev_bufs[b]
        return (fa2.kernel_fn(d["q"], d["k"], d["v"], causal=True, sm_scale=inp["sm_scale"]),)

    def download(b, outs):
        out_host[b].copy_(outs[0], non_blocking=True)

    total_s = time_pipelined(upload, compute, download, steps, warmup, device)
    return {"value": flops_total * steps / total_s / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": total_s / steps * 1e3, "pipelined": PIPELINE_NOTE}


def cpu_fa2_sample(s=8192, d=128, group=4, repeats=1):
    """The oracle (fp32 softmax(q k^T scale + causal mask) v, numpy) on the host cores over a sample
    of the FA2 workload: one (batch, key/value head) unit -- its `group` query heads over the full
    sequence; returns (TFLOP/s of the causal flop count, cores, seconds, sample text)."""
    sys.path.insert(0, ROOT)
    import oracle  # the CPU restatement; only this leg of the benchmark uses it

    gen = torch.Generator().manual_seed(3)
    q = torch.randn(1, group, s, d, generator=gen).to(torch.bfloat16).float().numpy()
    k = torch.randn(1, 1, s, d, generator=gen).to(torch.bfloat16).float().numpy()
    v = torch.randn(1, 1, s, d, generator=gen).to(torch.bfloat16).float().numpy()
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        oracle.fa2_attention(q, k, v, causal=True, sm_scale=1.0 / math.sqrt(d))
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    flops = fa2.get_flops(1, group, s, d, causal=True)
    return (flops / med / 1e12, os.cpu_count() or 1, med,
            f"one (batch, kv head) unit of the workload: {group} query heads x S={s} x D={d}, causal, fp32 "
            f"numpy oracle (oracle.fa2_attention) on the host cores, median of {repeats} ({med:.2f} s)")


def run_gdn_heads(device, rank, world, steps, warmup, verify=False):
    """GDN B1 T2048 strong-scaled: the 16 key heads (each with the value heads reading it) split
    across the ranks; every rank runs the whole 2048-token sequence for its heads."""
    full = gdn_inputs(device, 2048, seed=1000)
    ranges = sharding.even_ranges(HK, world)
    a, b = ranges[rank]
    inp = sharding.slice_gdn_inputs(full, a, b)
    if not verify:
        del full
    total_s, per = time_steps(lambda: gdn.kernel_fn(**inp), steps, warmup, device, flush=input_bytes(inp) < L2_BYTES)
    gdn.check_device_status(device)
    res = {"tokens_per_step": 2048, "ms": total_s / steps * 1e3, "value": 2048 * steps / total_s / 1e6,
           "unit": "Mtok/s", "kernel_ms_local": statistics.mean(per),
           "algo_bytes": gdn.algorithmic_bytes(2048, 1, hk=b - a, hv=2 * (b - a)), "token_heads": 2048 * 2 * (b - a),
           "schedule": gdn.schedule(inp["q"], inp["v"]),
           "config": {"workload": "gdn_b1_t2048_heads", "batch": 1, "seq_len": 2048, "hk": HK, "hv": HV,
                      "head_dim": D, "shard": f"key heads {HK // world}/rank (+ the value heads reading them)",
                      "scaling": "strong"}}
    if verify and world > 1:
        out, fs = gdn.kernel_fn(**inp)
        go = sharding.gather_to_rank0(out, dim=2)
        gs = sharding.gather_to_rank0(fs, dim=1)
        if rank == 0:
            ref_o, ref_s = gdn.kernel_fn(**full)
            sizes = [2 * (y - x) for x, y in ranges]
            offs = [sum(sizes[:i]) for i in range(world)]
            o = sharding.unscatter_gdn_heads([go.narrow(2, o0, n) for o0, n in zip(offs, sizes)], ranges, HK, HV, 2)
            st = sharding.unscatter_gdn_heads([gs.narrow(1, o0, n) for o0, n in zip(offs, sizes)], ranges, HK, HV, 1)
            res.update(compare_gdn(o, st, ref_o, ref_s))
    return res


HYBRID_B, HYBRID_HQ, HYBRID_HKV, HYBRID_D = 16, 16, 2, 256


def run_hybrid(device, rank, world, steps, warmup, seq_len):
    """The hybrid prefill sweep at one sequence length: FA2 causal GQA Hq=16 Hkv=2 D=256 and GDN
    prefill Hk=16 Hv=32 d=128, both over a batch of 16 sequences of `seq_len` tokens, the batch
    split evenly across the ranks (16 / N sequences per rank).  A step is one FA2 forward and one
    GDN prefill over the rank's sequences; each is also timed alone for its roofline."""
    local = HYBRID_B // world
    fi = fa2_inputs(device, local, HYBRID_HQ, HYBRID_HKV, seq_len, HYBRID_D, seed=40 + rank)
    gi = gdn_inputs(device, seq_len, seed=50 + rank, lengths=[seq_len] * local)
    flush = input_bytes(fi) + input_bytes(gi) < L2_BYTES
    fa_s, fa_per = time_steps(lambda: fa2.kernel_fn(**fi), steps, warmup, device, flush=flush)
    fa2.check_device_status(device)
    gd_s, gd_per = time_steps(lambda: gdn.kernel_fn(**gi), steps, warmup, device, flush=flush)
    gdn.check_device_status(device)

    def step():
        fa2.kernel_fn(**fi)
        gdn.kernel_fn(**gi)

    tot_s, per = time_steps(step, steps, warmup, device, flush=flush)
    tokens = HYBRID_B * seq_len
    fa_flops = fa2.get_flops(HYBRID_B, HYBRID_HQ, seq_len, HYBRID_D, causal=True)
    fa_local = fa2.get_flops(local, HYBRID_HQ, seq_len, HYBRID_D, causal=True)
    return {"tokens_per_step": tokens, "ms": tot_s / steps * 1e3, "value": tokens * steps / tot_s / 1e6,
            "unit": "Mtok/s", "kernel_ms_local": statistics.mean(per),
            "parts": {
                "fa2": {"ms": fa_s / steps * 1e3, "value": fa_flops * steps / fa_s / 1e12, "unit": "TFLOP/s",
                        "kernel_ms_local": statistics.mean(fa_per), "local_flops": fa_local,
                        "kernel": "tokmix::fa2::d256::fa2_fwd_d256_kernel"},
                "gdn": {"ms": gd_s / steps * 1e3, "value": tokens * steps / gd_s / 1e6, "unit": "Mtok/s",
                        "kernel_ms_local": statistics.mean(gd_per),
                        "algo_bytes": gdn.algorithmic_bytes(local * seq_len, local),
                        "token_heads": local * seq_len * HV,
                        "schedule": gdn.schedule(gi["q"], gi["v"], gi["cu_seqlens"])}},
            "config": {"workload": f"hybrid_t{seq_len}", "batch": HYBRID_B, "seq_len": seq_len,
                       "fa2": {"heads_q": HYBRID_HQ, "heads_kv": HYBRID_HKV, "head_dim": HYBRID_D, "causal": True},
                       "gdn": {"hk": HK, "hv": HV, "head_dim": D, "chunk": 64, "initial_state": "zero"},
                       "shard": f"batch {local}/rank", "l2": "flushed between timed steps" if flush
                       else "inputs larger than L2 (no flush)"}}


HYBRID_WORKLOADS = ["hybrid_t4096", "hybrid_t16384", "hybrid_t65536"]
# workloads that run on one GPU only (in "also" when the bench runs on one GPU)
ONE_GPU_WORKLOADS = list(ROW_OPS) + ["fa2_d256_b16_s4096"]


def e2e_gdn_b1(device, rank, world, steps, warmup, inp):
    """Headline step through the public plugin call from pinned host memory: every step uploads
    its inputs, runs kernel_fn and reads back the output and final state, pipelined as a serving
    loop runs it (time_pipelined)."""
    tensors = {k: v for k, v in inp.items() if isinstance(v, torch.Tensor)}
    host_arena, dev_arena, views = stage_arenas(tensors, device)
    dev_bufs = [views(a) for a in dev_arena]
    host = {"scale": inp["scale"]}
    out_host = [torch.empty((1, 2048, HV, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    st_host = [torch.empty((1, HV, D, D), dtype=torch.float32).pin_memory() for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in tensors.values())
    d2h = out_host[0].numel() * 2 + st_host[0].numel() * 4

    def upload(b):
        dev_arena[b].copy_(host_arena, non_blocking=True)

    def compute(b):
        args = dict(dev_bufs[b])
        args["scale"] = host["scale"]
        out, fs = gdn.kernel_fn(**args)
        return out, fs

    def download(b, outs):
        out_host[b].copy_(outs[0], non_blocking=True)
        st_host[b].copy_(outs[1], non_blocking=True)

    total_s = time_pipelined(upload, compute, download, steps, warmup, device)
    return {"value": 2048 * world * steps / total_s / 1e6, "unit": "Mtok/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": total_s / steps * 1e3, "pipelined": PIPELINE_NOTE}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_gdn_b1(repeats: int = 3):
    """The oracle (C restatement of the reference's fp32 recurrence) on the host cores, over the
    full B=1 T=2048 Hk=16 Hv=32 workload, `repeats` times; returns (Mtok/s median, cores, seconds)."""
    sys.path.insert(0, ROOT)
    import oracle  # the CPU restatement; only this leg of the benchmark uses it

    cores = os.cpu_count() or 1
    inp = gdn_inputs(torch.device("cpu"), 2048, seed=1000)
    args = [inp[k].float().numpy() for k in ("q", "k", "v", "g", "beta")]
    st = inp["state"].numpy()
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        oracle.gdn_recurrent(*args, st, inp["scale"], nthreads=cores)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return 2048 / med / 1e6, cores, med


def cpu_gdn_decode(batch: int = 128, repeats: int = 5):
    """The oracle on the host cores over the full decode workload (one token for each of `batch`
    sequences, Hk=16 Hv=32, N(0, 0.02) states); returns (Mtok/s median, cores, seconds)."""
    sys.path.insert(0, ROOT)
    import oracle  # the CPU restatement; only this leg of the benchmark uses it

    cores = os.cpu_count() or 1
    inp = gdn_dec.get_inputs(batch=batch, seed=5000, device="cpu")
    args = [inp[k].float().numpy() for k in ("q", "k", "v", "g", "beta")]
    st = inp["state"].numpy()
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        oracle.gdn_recurrent(*args, st, inp["scale"], nthreads=cores)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return batch / med / 1e6, cores, med


def run_reference(args):
    """`--impl reference`: the reference has no CPU implementation of this path (its oracle is a
    CUDA kernel), so the reference arm is the oracle port timed on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times = []
    cores = os.cpu_count() or 1
    for i in range(args.warmup + args.steps):
        v, cores, sec = cpu_gdn_b1(repeats=1)
        if i >= args.warmup:
            times.append(sec)
    total = sum(times)
    value = 2048 * args.steps / total / 1e6
    line = {"impl": "reference", "metric": HEADLINE_METRIC,
            "value": value, "unit": "Mtok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "Mtok/s", "cores": cores, "kind": "port",
                             "sample": "full B=1 T=2048 Hk=16 Hv=32 workload per step, fp32 recurrence "
                                       "(oracle/gdn_recurrent.c) on all host cores"},
            "e2e": {"value": value, "unit": "Mtok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="gdn_b1_t2048",
                    choices=["gdn_b1_t2048", "gdn_b1_t2048_heads", "fa2_b4_s8192", "gdn_varlen", "gdn_decode_b128",
                             "gdn_b4_t2048", "fa2_b1_s8192", "fa2_d256_b4_s4096"] + HYBRID_WORKLOADS
                            + ONE_GPU_WORKLOADS,
                    help="gdn_b4_t2048 / fa2_b1_s8192 / fa2_d256_b4_s4096 are profiling-size cases (inputs just above L2); the "
                         "row-wise op names time one op alone (one GPU); hybrid_t* run the hybrid prefill sweep")
    ap.add_argument("--no-also", action="store_true", help="skip the secondary workloads")
    ap.add_argument("--no-verify", action="store_true",
                    help="with N > 1, skip gathering the sharded outputs to rank 0 for comparison with a one-GPU run")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if world not in (1, 2, 4, 8):
        raise SystemExit("bench.py supports 1, 2, 4 or 8 GPUs")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    peaks = measured_peaks()
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    results = {}
    head = args.workload
    if (head in ONE_GPU_WORKLOADS or head == "fa2_d256_b4_s4096") and world != 1:
        raise SystemExit(f"workload {head} runs on one GPU")
    also = ["gdn_b1_t2048", "fa2_b4_s8192", "gdn_varlen", "gdn_decode_b128"] + (["gdn_b1_t2048_heads"] if world > 1 else [])
    order = [head] + ([w for w in also if w != head] if not args.no_also and head not in HYBRID_WORKLOADS else [])
    e2e = None
    for w in order:
        steps_w = args.steps if w == head else max(5, args.steps // 5)
        if w in ("gdn_b1_t2048", "gdn_b4_t2048"):
            r = run_gdn_batch(device, rank, world, steps_w, args.warmup, batch=1 if w == "gdn_b1_t2048" else 4)
            if w == head == "gdn_b1_t2048":
                e2e = e2e_gdn_b1(device, rank, world, args.steps, args.warmup, r["inp"])
            inp = r.pop("inp")
            r["config"] = headline_config(world) if w == "gdn_b1_t2048" else {
                "workload": w, "batch_per_rank": 4, "seq_len": 2048, "hk": HK, "hv": HV, "head_dim": D}
            del inp
        elif w in ("fa2_b4_s8192", "fa2_b1_s8192"):
            r = run_fa2(device, rank, world, steps_w, args.warmup, batch=4 if w == "fa2_b4_s8192" else 1,
                        verify=not args.no_verify, extras=(w == "fa2_b4_s8192"))
        elif w == "gdn_b1_t2048_heads":
            r = run_gdn_heads(device, rank, world, steps_w, args.warmup, verify=not args.no_verify)
        elif w in HYBRID_WORKLOADS:
            r = run_hybrid(device, rank, world, steps_w, args.warmup, seq_len=int(w[len("hybrid_t"):]))
        elif w == "gdn_decode_b128":
            r = run_gdn_decode(device, rank, world, steps_w, args.warmup)
        elif w in ROW_OPS:
            r = run_row_op(device, steps_w, args.warmup, w)
        elif w in ("fa2_d256_b16_s4096", "fa2_d256_b4_s4096"):
            r = run_fa2_d256(device, steps_w, args.warmup, batch=16 if w == "fa2_d256_b16_s4096" else 4)
        else:
            r = run_gdn_varlen(device, rank, world, steps_w, args.warmup, verify=not args.no_verify)
        results[w] = r
        torch.cuda.empty_cache()
    if world == 1 and not args.no_also and head not in HYBRID_WORKLOADS:
        for w in (x for x in ONE_GPU_WORKLOADS if x != head):
            steps_w = max(5, args.steps // 5)
            results[w] = (run_fa2_d256(device, steps_w, args.warmup) if w == "fa2_d256_b16_s4096"
                          else run_row_op(device, steps_w, args.warmup, w))
            torch.cuda.empty_cache()
    clocks = sampler.stop() if sampler else None

    cpu = None
    if rank == 0 and world == 1 and head == "gdn_decode_b128":
        v, cores, sec = cpu_gdn_decode()
        cpu = {"value": v, "unit": "Mtok/s", "cores": cores, "kind": "port",
               "sample": f"full decode step, 128 sequences Hk=16 Hv=32, median of 5 runs ({sec:.4f} s each), fp32 "
                         "recurrence (oracle/gdn_recurrent.c, OpenMP)"}
    elif rank == 0 and world == 1 and head in ("gdn_b1_t2048", "gdn_b1_t2048_heads", "gdn_b4_t2048", "gdn_varlen"):
        v, cores, sec = cpu_gdn_b1()
        cpu = {"value": v, "unit": "Mtok/s", "cores": cores, "kind": "port",
               "sample": f"full B=1 T=2048 Hk=16 Hv=32 workload, median of 3 runs ({sec:.3f} s each), fp32 "
                         "recurrence (oracle/gdn_recurrent.c, OpenMP)"}
    if rank == 0 and world == 1 and "fa2_b4_s8192" in results:
        v, cores, sec, sample = cpu_fa2_sample()
        fa2_cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}
        results["fa2_b4_s8192"]["cpu_baseline"] = fa2_cpu
        if head == "fa2_b4_s8192":
            cpu = fa2_cpu

    def roofline(w, r):
        if "parts" in r:  # hybrid sweep: one roofline per kernel
            return {"fa2": roofline("fa2_hybrid", r["parts"]["fa2"]), "gdn": roofline("gdn_hybrid", r["parts"]["gdn"])}
        kms = r["kernel_ms_local"]
        if w.startswith("fa2"):
            ach = r["local_flops"] / (kms / 1e3) / 1e12
            return {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": ach / peaks["bf16_tflops"], "peak_source": peaks["source"] + " burst bf16",
                    "frac_of_spec": ach / SPEC_BF16_TFLOPS,
                    "traffic": NCU_TRAFFIC_BYTES.get(w + "/fused"),
                    "kernel": r.get("kernel", "tokmix::fa2::fa2_fwd_kernel<128>"),
                    "kernel_ms": kms}
        ach = r["algo_bytes"] / (kms / 1e3) / 1e9
        if r.get("schedule") == "split":  # one step = the preparation launch + the state-chain launch
            kern = "tokmix::gdn::split::gdn_prep_kernel + tokmix::gdn::split::gdn_chain_kernel (one step)"
        elif r.get("schedule") == "overlap":  # one cooperative launch (after a memset of the record flags)
            kern = "tokmix::gdn::split::gdn_overlap_kernel"
        elif r.get("schedule") == "decode":
            kern = "tokmix::gdn_decode::gdn_decode_kernel"
        elif r.get("schedule") == "row_op":
            kern = r["kernel"]
        else:
            kern = "tokmix::gdn::gdn_prefill_kernel"
        line = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": ach / peaks["hbm_gbs"], "peak_source": peaks["source"] + " copy bandwidth",
                "frac_of_spec": ach / SPEC_HBM_GBS,
                "traffic": NCU_TRAFFIC_BYTES.get(f"{w}/{r.get('schedule', 'fused')}"), "algorithmic_bytes": r["algo_bytes"],
                "kernel": kern, "kernel_ms": kms, "schedule": r.get("schedule", "fused")}
        if "token_heads" in r:  # GDN: the tensor-core view of the same launch
            sec = kms / 1e3
            chunked = r["token_heads"] * GDN_CHUNKED_FLOP_PER_TOKEN_HEAD / sec / 1e12
            line["tensor"] = {"chunked_tflops": chunked, "chunked_frac": chunked / peaks["bf16_tflops"],
                              "flop_per_token_head": GDN_CHUNKED_FLOP_PER_TOKEN_HEAD,
                              "reference_formula_tflops": r["token_heads"] * 4 * D * D / sec / 1e12}
        return line

    if rank == 0:
        hr = results[head]
        metric = ("FA2 fwd TFLOPS" if head.startswith("fa2") else
                  "GDN decode Mtok/s" if head == "gdn_decode_b128" else
                  f"{ROW_OPS[head][1]} GB/s" if head in ROW_OPS else HEADLINE_METRIC)
        cfg = hr["config"]
        if head in HYBRID_WORKLOADS:
            metric = "hybrid prefill (FA2 D256 + GDN) Mtok/s"
            sched = hr["parts"]["gdn"]["schedule"]
            launches = args.steps * (1 + (2 if sched == "split" else 1))
        else:
            launches = args.steps * (2 if hr.get("schedule") == "split" else 1)
        if e2e is None and "e2e" in hr:
            e2e = hr["e2e"]
        extra_keys = ("verified_vs_one_gpu", "bitwise_vs_one_gpu", "max_abs_diff_vs_one_gpu", "e2e", "sdpa",
                      "cpu_baseline", "parts")
        line = {"metric": metric, "value": hr["value"], "unit": hr["unit"], "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": hr["ms"], "higher_is_better": True,
                "scaling": "weak" if head in ("gdn_b1_t2048", "gdn_b4_t2048") else "strong", "vs_baseline": None,
                "dtype": "bf16" if head.startswith("fa2") or head in ROW_OPS else "bf16 in / fp32 state",
                "data": "synthetic (seeded, B200 config shapes)", "config": cfg,
                "roofline": roofline(head, hr), "cpu_baseline": cpu,
                "e2e": e2e if e2e is not None else None,
                "gpu_launches": launches, "clocks": clocks,
                **({"sdpa": hr["sdpa"]} if "sdpa" in hr else {}),
                **({"parts": hr["parts"]} if "parts" in hr else {}),
                "also": {w: {"value": r["value"], "unit": r["unit"], "ms_per_step": r["ms"],
                             "roofline": roofline(w, r), **({"config": r["config"]} if "config" in r else {}),
                             **{x: r[x] for x in extra_keys if x in r}}
                         for w, r in results.items() if w != head}}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
