"""Same-box comparator: the reference's optimised sm_89 kernels (kernels_optimized/*.cu), recompiled
for sm_100a by oracle/build_ref.py, timed on one B200 beside this repository's kernels on the same
inputs.  COMPARISON INFRASTRUCTURE ONLY: nothing in the product imports this file.

Workloads are the shapes the reference kernels accept:
  fa2_b4_h32_s8192  causal attention B4 H32 S8192 D128, bf16, equal q/kv heads (the reference
                    rejects GQA, kernels_optimized/flash_attention_2.py:111-113); FLOPs by the
                    reference formula, kernel_configs/flash_attention_2.py:85-87
  gdn_b1_t{T}       GDN prefill B1 Hk16 Hv32 D128: the reference takes fp32 q/k/v/o
                    (kernels_optimized/qwen35moe_gdn_prefill.py:145-146), this repository bf16 q/k/v/o
                    with fp32 g/beta/state, both from the same draws

Each line is one JSON object: both implementations' device time per call (CUDA events, L2 flushed
between calls when the inputs fit in L2), their throughput, and the largest output difference.

    python oracle/time_ref_kernels.py [--steps 10 --warmup 3]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from kernel_opt_agent_b200 import flash_attention_2 as fa2  # noqa: E402
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn  # noqa: E402
from oracle.build_ref import load_built  # noqa: E402


def _time(fn, steps, warmup, device, flush):
    _, per = bench.time_steps(fn, steps, warmup, device, flush)
    return statistics.mean(per)


def compare_fa2(device, steps, warmup):
    ref = load_built("fa2_opt")
    B, H, S, Dh = 4, 32, 8192, 128
    inp = bench.fa2_inputs(device, B, H, H, S, Dh, seed=3)
    scale = inp["sm_scale"]
    flops = fa2.get_flops(B, H, S, Dh, causal=True)
    flush = bench.input_bytes(inp) < bench.L2_BYTES
    ms_ref = _time(lambda: ref.flash_attention_2_forward(inp["q"], inp["k"], inp["v"], scale, True),
                   steps, warmup, device, flush)
    ms_ours = _time(lambda: fa2.kernel_fn(**inp), steps, warmup, device, flush)
    o_ref = ref.flash_attention_2_forward(inp["q"], inp["k"], inp["v"], scale, True)
    o_ours = fa2.kernel_fn(**inp)
    diff = (o_ref.float() - o_ours.float()).abs().max().item()
    return {"workload": "fa2_b4_h32_s8192_d128_causal", "unit": "TFLOP/s",
            "reference_sm89_on_sm100a": {"ms": ms_ref, "value": flops / ms_ref / 1e9,
                                         "kernel": "kernels_optimized/flash_attention_2.cu (mma.sync)"},
            "this_repo": {"ms": ms_ours, "value": flops / ms_ours / 1e9, "kernel": "tokmix fa2_fwd_kernel (tcgen05)"},
            "speedup": ms_ref / ms_ours, "max_abs_diff_outputs": diff}


def compare_gdn(device, steps, warmup, tokens):
    ref = load_built("gdn_opt")
    inp = bench.gdn_inputs(device, tokens, seed=1)
    f32 = {k: (v.float() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    args = (f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], f32["state"], float(inp["scale"]))
    ms_ref = _time(lambda: ref.qwen35moe_gdn_prefill_bf16tc(*args), steps, warmup, device,
                   bench.input_bytes(f32) < bench.L2_BYTES)
    ms_ours = _time(lambda: gdn.kernel_fn(**inp), steps, warmup, device, bench.input_bytes(inp) < bench.L2_BYTES)
    o_ref, s_ref = ref.qwen35moe_gdn_prefill_bf16tc(*args)
    o_ours, s_ours = gdn.kernel_fn(**inp)
    return {"workload": f"gdn_b1_t{tokens}", "unit": "Mtok/s",
            "reference_sm89_on_sm100a": {"ms": ms_ref, "value": tokens / ms_ref / 1e3,
                                         "io": "fp32 q/k/v/o/g/beta/state",
                                         "kernel": "kernels_optimized/qwen35moe_gdn_prefill.cu (wmma, 2 launches)"},
            "this_repo": {"ms": ms_ours, "value": tokens / ms_ours / 1e3, "io": "bf16 q/k/v/o, fp32 g/beta/state",
                          "schedule": gdn.schedule(inp["q"], inp["v"])},
            "speedup": ms_ref / ms_ours,
            "max_abs_diff_out": (o_ref - o_ours.float()).abs().max().item(),
            "max_abs_diff_final_state": (s_ref - s_ours).abs().max().item()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", default="fa2,gdn")
    args = ap.parse_args()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    which = args.only.split(",")
    if "gdn" in which:
        for t in (2048, 8192):
            print(json.dumps(compare_gdn(device, args.steps, args.warmup, t)), flush=True)
    if "fa2" in which:
        print(json.dumps(compare_fa2(device, args.steps, args.warmup)), flush=True)


if __name__ == "__main__":
    main()
