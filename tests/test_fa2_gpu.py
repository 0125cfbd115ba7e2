"""FA2 parity on a B200: the sm_100a kernel (through the C ABI) against the fp32 oracle."""

import math
import pathlib

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import flash_attention_2 as fa2
from kernel_opt_agent_b200.kernel_configs import KERNEL_CONFIGS
from tests.golden import make_golden as golden

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
TOL = dict(atol=2e-2, rtol=2e-2)  # bf16 output tolerance


def _run_and_check(b, hq, hkv, s, d, causal, layout, seed=0, scale=None, tol=TOL):
    inp = fa2.get_inputs(b, hq, s, d, seed=seed, head_num_kv=hkv, layout=layout, causal=causal)
    if scale is not None:
        inp["sm_scale"] = scale
    out = fa2.kernel_fn(**inp)
    fa2.check_device_status(out.device)
    q, k, v = (inp[x].float().cpu().numpy() for x in ("q", "k", "v"))
    if layout == "bshd":
        q, k, v = (x.transpose(0, 2, 1, 3) for x in (q, k, v))
    ref = oracle.fa2_attention(q, k, v, causal=causal, sm_scale=inp["sm_scale"])
    got = out.float().cpu().numpy()
    if layout == "bshd":
        got = got.transpose(0, 2, 1, 3)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, **tol)
    return out


@pytest.mark.parametrize("b,hq,hkv,s,d,causal,layout", [
    (1, 2, 2, 128, 128, True, "bhsd"),
    (1, 2, 2, 129, 128, True, "bhsd"),
    (2, 4, 4, 257, 128, True, "bhsd"),
    (1, 4, 2, 200, 64, True, "bshd"),
    (1, 2, 1, 100, 128, False, "bhsd"),
    (1, 8, 8, 512, 64, True, "bshd"),      # B200 config 0 shape
    (1, 4, 4, 1031, 128, True, "bhsd"),
    (2, 6, 3, 300, 128, True, "bhsd"),
    (1, 3, 1, 256, 128, True, "bhsd"),      # odd group size: pairs of query tiles
    (1, 2, 2, 1, 128, True, "bhsd"),
    (1, 2, 2, 127, 64, False, "bhsd"),
    (1, 4, 1, 640, 128, False, "bshd"),
    (1, 2, 2, 128, 256, True, "bhsd"),      # head_dim 256: one query tile per CTA
    (1, 4, 1, 333, 256, True, "bhsd"),
    (2, 8, 1, 200, 256, True, "bshd"),      # config 4's 8:1 grouping
    (1, 2, 2, 65, 256, False, "bhsd"),
    (1, 2, 1, 1, 256, True, "bhsd"),
])
def test_fa2_matches_oracle(cuda_device, b, hq, hkv, s, d, causal, layout):
    _run_and_check(b, hq, hkv, s, d, causal, layout, seed=s + hq)


def test_fa2_custom_scale(cuda_device):
    _run_and_check(1, 2, 2, 300, 128, True, "bhsd", seed=3, scale=0.3)


@pytest.mark.parametrize("name", sorted(golden.FA2_CASES))
def test_fa2_matches_sdpa_golden(cuda_device, name):
    case = golden.FA2_CASES[name]
    q, k, v = (x.to(torch.bfloat16).to(cuda_device) for x in golden.fa2_inputs(case))
    out = fa2.kernel_fn(q, k, v, causal=case["causal"], layout=case["layout"])
    ref = np.load(GOLDEN / f"{name}.npz")["out_fp32"]
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, **TOL)


def test_fa2_stability_cases(cuda_device):
    cfg = KERNEL_CONFIGS["flash_attention_2"]
    size = {"batch": 1, "head_num": 4, "seq_len": 512, "head_dim": 128}
    for name, inp in cfg["numerical_stability_cases"](size, torch.bfloat16, "cuda"):
        out = fa2.kernel_fn(**inp)
        ref = cfg["reference_fn"](inp)
        assert torch.isfinite(out).all(), name
        torch.testing.assert_close(out.float(), ref.float(), atol=5e-2, rtol=5e-2, msg=name)


def test_fa2_config_sizes_against_sdpa(cuda_device):
    """Every toml test/edge size through the harness's own reference_fn (torch SDPA)."""
    cfg = KERNEL_CONFIGS["flash_attention_2"]
    tol = cfg["tolerances"][torch.bfloat16]
    for label, size in cfg["test_sizes"] + cfg["edge_sizes"]:
        inp = cfg["input_generator"](size, torch.bfloat16, "cuda", seed=42)
        out = fa2.kernel_fn(**inp)
        ref = cfg["reference_fn"](inp)
        torch.testing.assert_close(out.float(), ref.float(), **tol, msg=label)
        del inp, out, ref
    fa2.check_device_status(cuda_device)


def test_fa2_deterministic(cuda_device):
    inp = fa2.get_inputs(2, 8, 1000, 128, seed=9, head_num_kv=2)
    outs = [fa2.kernel_fn(**inp) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_fa2_full_size_gqa_sampled_rows(cuda_device):
    """B=4, Hq=32, Hkv=8, S=8192, D=128 causal: sampled query rows against the fp32 oracle."""
    inp = fa2.get_inputs(4, 32, 8192, 128, seed=0, head_num_kv=8)
    out = fa2.kernel_fn(**inp)
    fa2.check_device_status(cuda_device)
    rng = np.random.default_rng(0)
    rows = [(0, 0, 0), (3, 31, 8191), (1, 5, 127), (2, 17, 128), (0, 30, 4095), (1, 1, 4096)]
    rows += [(int(rng.integers(4)), int(rng.integers(32)), int(rng.integers(8192))) for _ in range(40)]
    for b, h, i in rows:
        q = inp["q"][b, h, i].float().cpu().numpy()
        kk = inp["k"][b, h // 4, : i + 1].float().cpu().numpy()
        vv = inp["v"][b, h // 4, : i + 1].float().cpu().numpy()
        s = kk @ q * inp["sm_scale"]
        p = np.exp(s - s.max())
        ref = (p @ vv) / p.sum()
        np.testing.assert_allclose(out[b, h, i].float().cpu().numpy(), ref, **TOL, err_msg=str((b, h, i)))


def test_fa2_hybrid_config_d256_sampled_rows(cuda_device):
    """The hybrid sweep's attention (Hq=16, Hkv=2, D=256, causal) at B=2 S=4096: sampled query
    rows against the fp32 oracle."""
    inp = fa2.get_inputs(2, 16, 4096, 256, seed=4, head_num_kv=2)
    out = fa2.kernel_fn(**inp)
    fa2.check_device_status(cuda_device)
    rng = np.random.default_rng(1)
    rows = [(0, 0, 0), (1, 15, 4095), (0, 7, 63), (1, 8, 64), (0, 3, 2047), (1, 12, 2048)]
    rows += [(int(rng.integers(2)), int(rng.integers(16)), int(rng.integers(4096))) for _ in range(30)]
    for b, h, i in rows:
        q = inp["q"][b, h, i].float().cpu().numpy()
        kk = inp["k"][b, h // 8, : i + 1].float().cpu().numpy()
        vv = inp["v"][b, h // 8, : i + 1].float().cpu().numpy()
        s = kk @ q * inp["sm_scale"]
        p = np.exp(s - s.max())
        ref = (p @ vv) / p.sum()
        np.testing.assert_allclose(out[b, h, i].float().cpu().numpy(), ref, **TOL, err_msg=str((b, h, i)))


def test_fa2_rejects_wrong_dtype(cuda_device):
    q = torch.zeros(1, 2, 64, 128, device=cuda_device)
    with pytest.raises(ValueError):
        fa2.kernel_fn(q, q, q)
    q = torch.zeros(1, 2, 64, 96, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fa2.kernel_fn(q, q, q)
