"""Generates the golden vectors under tests/golden/ (committed together with this script).

  python tests/golden/make_golden.py --fa2 [--out DIR]   # CPU: torch's own SDPA (the reference's FA2 oracle)
  python tests/golden/make_golden.py --gdn [--out DIR]   # B200: the reference's scalar GDN CUDA kernel
  python tests/golden/make_golden.py --rowops [--reference DIR] [--out DIR]
                                                         # CPU: the reference's row-op checkers

FA2: the reference's oracle is ``torch.nn.functional.scaled_dot_product_attention``
(``references/flash_attention_2.py:33-41``); it is run here on the CPU in fp32 from bf16-rounded
inputs.  GDN: the reference's oracle is its fp32 scalar CUDA kernel
(``kernels/qwen35moe_gdn_prefill.cu:31-100``), built from the reference sources by
``oracle/build_ref.py`` and run on a B200.  Inputs are not stored: they are regenerated from
the formulas/seeds in ``golden_inputs`` below, which the tests import.  To keep the files small
only some heads of each output are stored.  Row ops: the reference's own torch checkers
(``references/{rms_norm,swiglu_input_quant,qkv_part_rope}.py``), loaded from the reference
checkout and run here on the CPU; every output is stored bit for bit (bf16 / fp16 / e4m3 as raw
integers), so that the repository's checkers can be pinned without the checkout.
"""

from __future__ import annotations

import argparse
import json
import math
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

GDN_OUT_HEADS = [0, 1, 16, 17, 31]
GDN_STATE_HEADS = [0, 17, 31]

FA2_CASES = {
    "fa2_s129_d128_causal": dict(b=1, hq=2, hkv=2, s=129, d=128, causal=True, layout="bhsd", seed=11),
    "fa2_s200_d64_gqa_bshd": dict(b=1, hq=4, hkv=2, s=200, d=64, causal=True, layout="bshd", seed=12),
    "fa2_s100_d128_noncausal": dict(b=1, hq=2, hkv=1, s=100, d=128, causal=False, layout="bhsd", seed=13),
}

GDN_CASES = {
    "gdn_fixture_t67": dict(kind="fixture", t=67),
    "gdn_random_t96_state": dict(kind="random", t=96, seed=7, state_std=0.02),
    "gdn_strong_gate_t64": dict(kind="strong_gate", t=64, seed=3),
}


def _bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def fa2_inputs(case: dict):
    """bf16-representable q, k, v (as fp32 tensors, layout of the case)."""
    gen = torch.Generator().manual_seed(case["seed"])
    b, hq, hkv, s, d = case["b"], case["hq"], case["hkv"], case["s"], case["d"]

    def shape(h):
        return (b, h, s, d) if case["layout"] == "bhsd" else (b, s, h, d)

    q = _bf16_round(torch.randn(shape(hq), generator=gen))
    k = _bf16_round(torch.randn(shape(hkv), generator=gen))
    v = _bf16_round(torch.randn(shape(hkv), generator=gen))
    return q, k, v


def gdn_inputs(case: dict):
    """fp32 tensors q,k [1,T,16,128], v [1,T,32,128], g, beta [1,T,32], state [1,32,128,128]."""
    t = case["t"]
    if case["kind"] == "fixture":
        def filled(shape, scale, bias):
            n = int(np.prod(shape))
            x = torch.arange(n, dtype=torch.float32)
            return (((x % 251) - 125.0) * scale + bias).reshape(shape)
        return (filled((1, t, 16, 128), 1e-3, 0.0), filled((1, t, 16, 128), 1e-3, 0.0),
                filled((1, t, 32, 128), 1e-3, 0.0), filled((1, t, 32), 1e-4, -0.01),
                filled((1, t, 32), 1e-4, 0.5), filled((1, 32, 128, 128), 1e-4, 0.0))
    gen = torch.Generator().manual_seed(case["seed"])
    q = torch.randn(1, t, 16, 128, generator=gen)
    k = torch.randn(1, t, 16, 128, generator=gen)
    q = _bf16_round(q / q.norm(dim=-1, keepdim=True))
    k = _bf16_round(k / k.norm(dim=-1, keepdim=True))
    v = _bf16_round(torch.randn(1, t, 32, 128, generator=gen))
    g = -torch.nn.functional.softplus(torch.randn(1, t, 32, generator=gen))
    beta = torch.sigmoid(torch.randn(1, t, 32, generator=gen))
    state = torch.randn(1, 32, 128, 128, generator=gen) * case.get("state_std", 0.0)
    if case["kind"] == "strong_gate":
        g = torch.rand(1, t, 32, generator=gen) * 17.0 - 25.0
    return q, k, v, g, beta, state


def make_fa2(out_dir: pathlib.Path):
    import torch.nn.functional as F

    for name, case in FA2_CASES.items():
        q, k, v = fa2_inputs(case)
        if case["layout"] == "bshd":
            q, k, v = (x.transpose(1, 2) for x in (q, k, v))
        scale = 1.0 / math.sqrt(case["d"])
        o32 = F.scaled_dot_product_attention(q, k, v, is_causal=case["causal"], scale=scale,
                                             enable_gqa=case["hq"] != case["hkv"])
        o16 = F.scaled_dot_product_attention(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16),
                                             is_causal=case["causal"], scale=scale,
                                             enable_gqa=case["hq"] != case["hkv"]).float()
        if case["layout"] == "bshd":
            o32, o16 = o32.transpose(1, 2), o16.transpose(1, 2)
        np.savez_compressed(out_dir / f"{name}.npz", out_fp32=o32.contiguous().numpy(),
                            out_sdpa_bf16=o16.contiguous().numpy())
        print("wrote", name)


def make_gdn(out_dir: pathlib.Path):
    sys.path.insert(0, str(ROOT))
    from oracle.build_ref import load_built

    ext = load_built()
    dev = torch.device("cuda", 0)
    for name, case in GDN_CASES.items():
        q, k, v, g, beta, state = (x.to(dev).contiguous() for x in gdn_inputs(case))
        out, fs = ext.qwen35moe_gdn_prefill_ref(q, k, v, g, beta, state, 128 ** -0.5)
        torch.cuda.synchronize()
        np.savez_compressed(out_dir / f"{name}.npz", out=out[:, :, GDN_OUT_HEADS].cpu().numpy(),
                            final_state=fs[:, GDN_STATE_HEADS].cpu().numpy())
        print("wrote", name)
    meta = {"device": torch.cuda.get_device_name(0), "torch": torch.__version__,
            "out_heads": GDN_OUT_HEADS, "state_heads": GDN_STATE_HEADS}
    (out_dir / "gdn_golden_meta.json").write_text(json.dumps(meta, indent=1))


ROWOP_CASES = {
    "rowop_rms_norm_bf16": dict(op="rms_norm", m=64, n=512, dtype="bfloat16", seed=31),
    "rowop_rms_norm_fp16": dict(op="rms_norm", m=33, n=1040, dtype="float16", seed=32),
    "rowop_swiglu_quant": dict(op="swiglu_input_quant", m=48, n=384, seed=33),
    "rowop_rope": dict(op="qkv_part_rope", b=1, s=16, heads=12, d=256, q_heads=10, kv_heads=1, nope=192,
                       negative_sin=False, seed=34),
    "rowop_rope_negsin": dict(op="qkv_part_rope", b=1, s=17, heads=6, d=128, q_heads=3, kv_heads=2, nope=64,
                              negative_sin=True, seed=35),
}


def rowop_inputs(case: dict) -> dict:
    """Seeded CPU inputs of a row-op case (the keyword arguments of its checker)."""
    gen = torch.Generator().manual_seed(case["seed"])
    if case["op"] == "rms_norm":
        dt = getattr(torch, case["dtype"])
        x = (torch.randn(case["m"], case["n"], generator=gen) * 2.0).to(dt)
        w = (torch.rand(case["n"], generator=gen) + 0.5).to(dt)
        return {"x": x, "weight": w, "eps": 1e-6}
    if case["op"] == "swiglu_input_quant":
        x = (torch.randn(case["m"], 2 * case["n"], generator=gen) * 3.0).to(torch.bfloat16)
        x[0, :128] = 0.0  # an all-zero block: the eps clamp
        return {"x": x}
    rope = case["d"] - case["nope"]
    pos = torch.arange(case["s"], dtype=torch.float32)[:, None]
    inv = 10000.0 ** (-torch.arange(0, rope, 2, dtype=torch.float32) / rope)
    return {"qkv": torch.randn(case["b"], case["s"], case["heads"], case["d"], generator=gen).to(torch.bfloat16),
            "cos": torch.cos(pos * inv), "sin": torch.sin(pos * inv), "q_heads": case["q_heads"],
            "kv_heads": case["kv_heads"], "nope_dim": case["nope"], "negative_sin": case["negative_sin"]}


def raw(t: torch.Tensor) -> np.ndarray:
    """The tensor's bits as an integer array (2- or 1-byte types) or its fp32 values."""
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy()
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy()
    return t.contiguous().numpy()


def reference_rowop_checkers(reference: pathlib.Path) -> dict:
    """The reference's three row-op checker functions, loaded file by file from its checkout."""
    import importlib.util

    fns = {}
    for op in ("rms_norm", "swiglu_input_quant", "qkv_part_rope"):
        spec = importlib.util.spec_from_file_location(f"_ref_{op}", reference / "references" / f"{op}.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        fns[op] = getattr(mod, f"{op}_ref")
    return fns


def make_rowops(out_dir: pathlib.Path, reference: pathlib.Path):
    fns = reference_rowop_checkers(reference)
    for name, case in ROWOP_CASES.items():
        res = fns[case["op"]](**rowop_inputs(case))
        res = res if isinstance(res, tuple) else (res,)
        np.savez_compressed(out_dir / f"{name}.npz", **{f"out{i}": raw(t) for i, t in enumerate(res)})
        print("wrote", name)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--fa2", action="store_true")
    ap.add_argument("--gdn", action="store_true")
    ap.add_argument("--rowops", action="store_true")
    ap.add_argument("--reference", type=pathlib.Path, default=pathlib.Path("/root/reference"))
    ap.add_argument("--out", type=pathlib.Path, default=HERE)
    a = ap.parse_args()
    a.out.mkdir(parents=True, exist_ok=True)
    if a.fa2:
        make_fa2(a.out)
    if a.gdn:
        make_gdn(a.out)
    if a.rowops:
        make_rowops(a.out, a.reference)
