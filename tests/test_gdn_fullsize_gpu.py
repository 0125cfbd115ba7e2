"""GDN prefill parity at full size on a B200: long sequences and the configured workloads against
the fp32 recurrence oracle (``kernels/qwen35moe_gdn_prefill.cu:55-99`` restated in
``oracle/gdn_recurrent.c``), every sequence and every head compared.

The kernels keep the fp32 state in tensor memory and feed the state products hi+lo bf16 splits,
so these cases check that the state holds the fp32 tolerance over hundreds to a thousand 64-token
chunks: the varlen workload's eight sequences (up to 347 chunks), the reference's configured
lengths (``kernel_configs/qwen35moe_gdn_prefill.toml:5-33``: 4096, 8192, 4097, 8191) through its
fp32 fixture and through the random workload, and the hybrid sweep's sequence lengths 16384 and
65536 (256 and 1024 chunks) under every schedule.

With TOKMIX_PARITY_REPORT=<path> each case appends one JSON line with its worst errors (the
largest absolute error and the largest fraction of the tolerance used, for output and state).
"""

import json
import os

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import KERNEL_CONFIGS
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=2e-2, rtol=2e-2)     # bf16 output
STATE_TOL = dict(atol=1e-4, rtol=1e-3)   # fp32 final state


def _np(x):
    return None if x is None else x.float().cpu().numpy()


def _oracle(inp, threads):
    return oracle.gdn_recurrent(_np(inp["q"]), _np(inp["k"]), _np(inp["v"]), _np(inp["g"]), _np(inp["beta"]),
                                _np(inp.get("state")), inp.get("scale"), cu_seqlens=_np(inp.get("cu_seqlens")),
                                nthreads=threads)


def _errors(got, ref, tol):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    used = err / (tol["atol"] + tol["rtol"] * np.abs(ref.astype(np.float64)))
    return float(err.max(initial=0.0)), float(used.max(initial=0.0))


def _report(case, out_err, state_err):
    path = os.environ.get("TOKMIX_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": case, "out_max_abs": out_err[0], "out_tol_used": out_err[1],
                                "state_max_abs": state_err[0], "state_tol_used": state_err[1]}) + "\n")


def _compare(case, got_o, got_s, ref_o, ref_s, out_tol=OUT_TOL, state_tol=STATE_TOL):
    assert np.isfinite(got_o).all() and np.isfinite(got_s).all(), case
    ref_s = ref_s.reshape(got_s.shape)
    _report(case, _errors(got_o, ref_o, out_tol), _errors(got_s, ref_s, state_tol))
    np.testing.assert_allclose(got_o, ref_o, **out_tol, err_msg=case)
    np.testing.assert_allclose(got_s, ref_s, **state_tol, err_msg=case)


def test_gdn_varlen_every_sequence_matches_oracle(cuda_device, oracle_threads):
    """The packed varlen workload: 8 sequences of U[1024, 32768] tokens (117,560 in all), initial
    states N(0, 0.02); every sequence's output and final state against the oracle."""
    lengths = gcfg.varlen_lengths(8, seed=0)
    inp = gcfg.random_inputs(1, 0, lengths=lengths, seed=0, state_std=0.02)
    out, fs = gdn.kernel_fn(**inp)
    gdn.check_device_status(cuda_device)
    ref_o, ref_s = _oracle(inp, oracle_threads)
    _compare(f"varlen8 {gdn.schedule(inp['q'], inp['v'], inp['cu_seqlens'])}", _np(out), _np(fs), ref_o, ref_s)


@pytest.mark.parametrize("t", [4096, 8192, 4097, 8191])
def test_gdn_reference_fixture_configured_lengths(cuda_device, oracle_threads, t):
    """The reference's deterministic fixture through its fp32 interface at its configured lengths,
    at its own fp32 tolerance."""
    tol = KERNEL_CONFIGS["qwen35moe_gdn_prefill"]["tolerances"][torch.float32]
    inp = gcfg.fixture_inputs(1, t, torch.float32, "cuda")
    out, fs = gdn.kernel_fn(**inp)
    gdn.check_device_status(cuda_device)
    assert out.dtype == torch.float32
    ref_o, ref_s = _oracle(inp, oracle_threads)
    _compare(f"fixture fp32 T{t}", _np(out), _np(fs), ref_o, ref_s, out_tol=tol, state_tol=tol)


@pytest.mark.parametrize("t", [4096, 8192, 4097, 8191])
def test_gdn_random_workload_configured_lengths(cuda_device, oracle_threads, t):
    """The random workload (bf16 q/k/v, fp32 gates and state) at the configured lengths."""
    inp = gcfg.random_inputs(1, t, seed=t, state_std=0.02)
    out, fs = gdn.kernel_fn(**inp)
    gdn.check_device_status(cuda_device)
    ref_o, ref_s = _oracle(inp, oracle_threads)
    _compare(f"random T{t} {gdn.schedule(inp['q'], inp['v'])}", _np(out), _np(fs), ref_o, ref_s)


@pytest.fixture(scope="module")
def long16k():
    inp = gcfg.random_inputs(1, 16384, seed=16384, state_std=0.02)
    return inp, _oracle(inp, os.cpu_count() or 1)


@pytest.mark.parametrize("mode", ["auto", "fused", "split", "overlap", "segmented"])
def test_gdn_long_sequence_16k(cuda_device, long16k, mode):
    """One sequence of 16384 tokens (256 chunks), every head, under each schedule."""
    inp, (ref_o, ref_s) = long16k
    out, fs = gdn.kernel_fn(**inp, mode=mode)
    gdn.check_device_status(cuda_device)
    name = gdn.schedule(inp["q"], inp["v"], mode=mode)
    _compare(f"long T16384 {mode}->{name}", _np(out), _np(fs), ref_o, ref_s)


@pytest.fixture(scope="module")
def long64k():
    inp = gcfg.random_inputs(1, 65536, seed=65536, state_std=0.02)
    return inp, _oracle(inp, os.cpu_count() or 1)


@pytest.mark.parametrize("mode", ["auto", "fused", "split", "overlap", "segmented"])
def test_gdn_long_sequence_64k(cuda_device, long64k, mode):
    """One sequence of 65536 tokens (1024 chunks), every head: the hybrid sweep's longest length."""
    inp, (ref_o, ref_s) = long64k
    out, fs = gdn.kernel_fn(**inp, mode=mode)
    gdn.check_device_status(cuda_device)
    name = gdn.schedule(inp["q"], inp["v"], mode=mode)
    _compare(f"long T65536 {mode}->{name}", _np(out), _np(fs), ref_o, ref_s)


def test_gdn_weak_decay_long_sequence(cuda_device, oracle_threads):
    """Weak decay (g = -0.002 per token, the state keeps ~88 % per chunk) over 8192 tokens: the case
    in which rounding in the state path accumulates longest."""
    inp = gcfg.random_inputs(1, 8192, seed=77, state_std=0.02, hk=4, hv=8)
    inp["g"] = torch.full_like(inp["g"], -0.002)
    for mode in ("fused", "split"):
        out, fs = gdn.kernel_fn(**inp, mode=mode)
        gdn.check_device_status(cuda_device)
        ref_o, ref_s = _oracle(inp, oracle_threads)
        _compare(f"weak decay T8192 {mode}", _np(out), _np(fs), ref_o, ref_s)
