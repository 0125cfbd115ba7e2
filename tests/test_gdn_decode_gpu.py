"""GDN decode step on a B200: tokmix_gdn_decode (through the C ABI) against the fp32 recurrence
oracle for one token, and against the prefill kernel for a token-by-token sequence."""

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import qwen35moe_gdn_decode as dec
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=2e-2, rtol=2e-2)     # bf16 output
STATE_TOL = dict(atol=1e-4, rtol=1e-3)   # fp32 final state


def _np(x):
    return None if x is None else x.float().cpu().numpy()


def _oracle(inp, threads):
    return oracle.gdn_recurrent(_np(inp["q"]), _np(inp["k"]), _np(inp["v"]), _np(inp["g"]), _np(inp["beta"]),
                                _np(inp.get("state")), inp.get("scale"), nthreads=threads)


@pytest.mark.parametrize("b,hk,hv,state_std", [
    (1, 16, 32, 0.0),
    (1, 16, 32, 0.02),
    (3, 2, 4, 0.02),
    (5, 1, 1, 0.5),
    (64, 16, 32, 0.02),
    (7, 4, 8, 0.02),
])
def test_decode_matches_oracle(cuda_device, oracle_threads, b, hk, hv, state_std):
    inp = gcfg.random_inputs(b, 1, seed=100 + b + hv, state_std=state_std, hk=hk, hv=hv)
    out, fs = dec.kernel_fn(**inp)
    o_ref, s_ref = _oracle(inp, oracle_threads)
    assert torch.isfinite(out.float()).all() and torch.isfinite(fs).all()
    np.testing.assert_allclose(_np(out), o_ref, **OUT_TOL)
    np.testing.assert_allclose(_np(fs), s_ref, **STATE_TOL)


def test_decode_zero_state_and_none_agree(cuda_device):
    inp = gcfg.random_inputs(4, 1, seed=3, state_std=0.0)
    a = dec.kernel_fn(**inp)
    inp["state"] = None
    b = dec.kernel_fn(**inp)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_decode_inplace_is_bitwise_out_of_place(cuda_device):
    inp = gcfg.random_inputs(8, 1, seed=4, state_std=0.02)
    ref_o, ref_s = dec.kernel_fn(**inp)
    st = inp["state"].clone()
    o, s = dec.kernel_fn(**{**inp, "state": st}, inplace=True)
    assert s.data_ptr() == st.data_ptr()
    assert torch.equal(o, ref_o) and torch.equal(st, ref_s)


def test_decode_loop_equals_prefill_and_oracle(cuda_device, oracle_threads):
    """T decode steps (state updated in place) reproduce the prefill of the whole sequence."""
    T = 24
    inp = gcfg.random_inputs(2, T, seed=9, state_std=0.02, hk=2, hv=4)
    st = inp["state"].clone()
    outs = []
    for t in range(T):
        step = {n: inp[n][:, t:t + 1] for n in ("q", "k", "v", "g", "beta")}
        o, _ = dec.kernel_fn(**step, state=st, scale=inp["scale"], inplace=True)
        outs.append(o)
    out = torch.cat(outs, dim=1)
    o_ref, s_ref = _oracle(inp, oracle_threads)
    np.testing.assert_allclose(_np(out), o_ref, **OUT_TOL)
    np.testing.assert_allclose(_np(st), s_ref, **STATE_TOL)
    p_out, p_state = gdn.kernel_fn(**inp)
    np.testing.assert_allclose(_np(st), _np(p_state), **STATE_TOL)
    np.testing.assert_allclose(_np(out), _np(p_out), **OUT_TOL)


def test_decode_fp32_interface(cuda_device, oracle_threads):
    """The reference's all-fp32 tensors: q/k/v rounded to bf16 on the device, fp32 output."""
    inp = gcfg.random_inputs(3, 1, dtype=torch.float32, seed=11, state_std=0.02)
    out, fs = dec.kernel_fn(**inp)
    assert out.dtype == torch.float32
    rounded = {n: (inp[n].to(torch.bfloat16) if n in ("q", "k", "v") else inp[n]) for n in inp}
    o_ref, s_ref = _oracle(rounded, oracle_threads)
    np.testing.assert_allclose(_np(out), o_ref, **OUT_TOL)
    np.testing.assert_allclose(_np(fs), s_ref, **STATE_TOL)


def test_decode_rejects_bad_shapes(cuda_device):
    inp = gcfg.random_inputs(2, 2, seed=1)
    with pytest.raises(ValueError):
        dec.kernel_fn(**inp)  # two tokens
    inp = gcfg.random_inputs(2, 1, seed=1)
    with pytest.raises(ValueError):
        dec.kernel_fn(**{**inp, "state": inp["state"][:1]})
    with pytest.raises(ValueError):
        dec.kernel_fn(**{**inp, "state": None}, inplace=True)


def test_decode_empty_batch(cuda_device):
    inp = gcfg.random_inputs(1, 1, seed=2)
    empty = {n: (v[:0] if isinstance(v, torch.Tensor) else v) for n, v in inp.items()}
    out, fs = dec.kernel_fn(**empty)
    assert out.shape[0] == 0 and fs.shape[0] == 0


def test_decode_config_sizes_against_config_reference(cuda_device):
    """Every size of kernel_configs/qwen35moe_gdn_decode.toml through the config's own generator
    and checker (the harness's path), at the config's tolerance for each dtype."""
    from kernel_opt_agent_b200.kernel_configs import KERNEL_CONFIGS

    cfg = KERNEL_CONFIGS["qwen35moe_gdn_decode"]
    for dtype in cfg["test_dtypes"]:
        tol = cfg["tolerances"][dtype]
        for label, size in cfg["test_sizes"] + cfg["edge_sizes"]:
            inp = cfg["input_generator"](size, dtype, "cuda")
            out, fs = dec.kernel_fn(**inp)
            ref_o, ref_s = cfg["reference_fn"](inp)
            torch.testing.assert_close(out.float(), ref_o.float(), **tol, msg=lambda m: f"{label} {dtype}: {m}")
            # bf16 inputs: the checker sees the kernel's operands, so the fp32 state must agree to
            # the strict state tolerance; fp32 inputs are rounded to bf16 by the kernel only, so
            # the config's fp32 tolerance applies to both outputs, as in the harness
            state_tol = dict(atol=1e-4, rtol=1e-3) if dtype == torch.bfloat16 else tol
            torch.testing.assert_close(fs, ref_s, **state_tol, msg=lambda m: f"{label} {dtype}: {m}")
