"""GDN prefill parity on a B200: the sm_100a chunked kernel (through the C ABI) against the
fp32 recurrence oracle."""

import json
import pathlib

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import KERNEL_CONFIGS
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg
from tests.golden import make_golden as golden

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
OUT_TOL = dict(atol=2e-2, rtol=2e-2)     # bf16 output
STATE_TOL = dict(atol=1e-4, rtol=1e-3)   # fp32 final state


def _np(x):
    return None if x is None else x.float().cpu().numpy()


def _oracle(inp, threads):
    return oracle.gdn_recurrent(_np(inp["q"]), _np(inp["k"]), _np(inp["v"]), _np(inp["g"]), _np(inp["beta"]),
                                _np(inp.get("state")), inp.get("scale"), cu_seqlens=_np(inp.get("cu_seqlens")),
                                nthreads=threads)


def _check(inp, threads, out_tol=OUT_TOL, state_tol=STATE_TOL, mode="auto"):
    out, fs = gdn.kernel_fn(**inp, mode=mode)
    gdn.check_device_status(out.device)
    o_ref, s_ref = _oracle(inp, threads)
    got_o, got_s = _np(out), _np(fs)
    assert np.isfinite(got_o).all() and np.isfinite(got_s).all()
    np.testing.assert_allclose(got_o, o_ref, **out_tol)
    np.testing.assert_allclose(got_s, s_ref.reshape(got_s.shape), **state_tol)
    return out, fs


@pytest.mark.parametrize("b,t,hk,hv,state_std", [
    (1, 1, 16, 32, 0.0),
    (1, 2, 2, 4, 0.02),
    (1, 63, 2, 4, 0.0),
    (1, 64, 2, 4, 0.02),
    (2, 65, 2, 4, 0.02),
    (1, 128, 1, 1, 0.0),
    (1, 200, 16, 32, 0.02),
    (3, 129, 4, 8, 0.02),
])
def test_gdn_matches_oracle(cuda_device, oracle_threads, b, t, hk, hv, state_std):
    inp = gcfg.random_inputs(b, t, seed=t + hk, state_std=state_std, hk=hk, hv=hv)
    _check(inp, oracle_threads)


def test_gdn_varlen_with_empty_and_tail_sequences(cuda_device, oracle_threads):
    inp = gcfg.random_inputs(1, 0, lengths=[1, 63, 64, 65, 200, 0, 129], seed=5, state_std=0.02)
    _check(inp, oracle_threads)


# Both schedules (one CTA per unit; chunk-parallel preparation + state-chain launch) on the same
# inputs: each against the oracle, and against each other.
@pytest.mark.parametrize("mode", ["fused", "split", "overlap"])
@pytest.mark.parametrize("b,t,hk,hv,state_std,lengths", [
    (1, 1, 16, 32, 0.0, None),
    (2, 65, 2, 4, 0.02, None),
    (3, 129, 4, 8, 0.02, None),
    (1, 0, 2, 4, 0.02, [1, 63, 64, 65, 200, 0, 129]),
])
def test_gdn_schedules_match_oracle(cuda_device, oracle_threads, mode, b, t, hk, hv, state_std, lengths):
    inp = gcfg.random_inputs(b, t, seed=t + hk + 1, state_std=state_std, hk=hk, hv=hv, lengths=lengths)
    _check(inp, oracle_threads, mode=mode)


def test_gdn_schedules_agree_bitwise(cuda_device):
    """The three schedules issue the same operations in the same order: identical results."""
    inp = gcfg.random_inputs(2, 300, seed=9, state_std=0.02, hk=4, hv=8)
    o1, s1 = gdn.kernel_fn(**inp, mode="fused")
    for mode in ("split", "overlap"):
        o2, s2 = gdn.kernel_fn(**inp, mode=mode)
        assert torch.equal(o1, o2) and torch.equal(s1, s2), mode


def test_gdn_reference_fixture_fp32_io(cuda_device, oracle_threads):
    """The reference's own fixture and fp32 interface, at its own tolerance."""
    cfg = KERNEL_CONFIGS["qwen35moe_gdn_prefill"]
    tol = cfg["tolerances"][torch.float32]
    for t in (2048, 2113):
        inp = gcfg.fixture_inputs(1, t, torch.float32, "cuda")
        out, fs = gdn.kernel_fn(**inp)
        assert out.dtype == torch.float32
        o_ref, s_ref = _oracle(inp, oracle_threads)
        np.testing.assert_allclose(_np(out), o_ref, **tol)
        np.testing.assert_allclose(_np(fs), s_ref, **tol)


def test_gdn_stability_cases(cuda_device, oracle_threads):
    cfg = KERNEL_CONFIGS["qwen35moe_gdn_prefill"]
    for name, inp in cfg["numerical_stability_cases"]({"batch": 1, "seq_len": 300, "dist": "random"},
                                                       torch.bfloat16, "cuda"):
        out, fs = gdn.kernel_fn(**inp)
        o_ref, s_ref = _oracle(inp, oracle_threads)
        # the reference relaxes its tolerance x10 for these cases (tools/bench.py:557-609)
        np.testing.assert_allclose(_np(out), o_ref, atol=2e-2, rtol=2e-2, err_msg=name)
        np.testing.assert_allclose(_np(fs), s_ref, atol=1e-3, rtol=1e-2, err_msg=name)


def test_gdn_strong_negative_gate_strict(cuda_device, oracle_threads):
    inp = gcfg.random_inputs(1, 64, seed=3)
    gen = torch.Generator().manual_seed(4)
    inp["g"] = (torch.rand(inp["g"].shape, generator=gen) * 17.0 - 25.0).cuda()
    _check(inp, oracle_threads)


@pytest.mark.skipif(not (GOLDEN / "gdn_golden_meta.json").exists(), reason="GDN golden vectors not generated")
@pytest.mark.parametrize("name", sorted(golden.GDN_CASES))
def test_gdn_matches_reference_kernel_golden(cuda_device, name):
    meta = json.loads((GOLDEN / "gdn_golden_meta.json").read_text())
    case = golden.GDN_CASES[name]
    q, k, v, g, beta, st = (x.cuda() for x in golden.gdn_inputs(case))
    io = torch.float32 if case["kind"] == "fixture" else torch.bfloat16
    out, fs = gdn.kernel_fn(q.to(io), k.to(io), v.to(io), g, beta, st)
    ref = np.load(GOLDEN / f"{name}.npz")
    tol_o = dict(atol=2e-3, rtol=2e-1) if case["kind"] == "fixture" else OUT_TOL
    tol_s = dict(atol=2e-3, rtol=2e-1) if case["kind"] == "fixture" else STATE_TOL
    np.testing.assert_allclose(_np(out)[:, :, meta["out_heads"]], ref["out"], **tol_o)
    np.testing.assert_allclose(_np(fs)[:, meta["state_heads"]], ref["final_state"], **tol_s)


@pytest.mark.parametrize("mode", ["fused", "split", "overlap"])
def test_gdn_config1_full(cuda_device, oracle_threads, mode):
    """B=1, T=2048, Hk=16, Hv=32, zero state: every output and the fp32 final state."""
    inp = gcfg.random_inputs(1, 2048, seed=0)
    _check(inp, oracle_threads, mode=mode)


def test_gdn_state_continuation_is_exact(cuda_device):
    """Chunk-aligned split with the state handed over equals the one-shot run bit for bit."""
    inp = gcfg.random_inputs(1, 640, seed=8, state_std=0.02)
    out, fs = gdn.kernel_fn(**inp, mode="split")
    a = {k: (v[:, :256] if k in ("q", "k", "v", "g", "beta") else v) for k, v in inp.items()}
    oa, sa = gdn.kernel_fn(**a, mode="split")
    b = {k: (v[:, 256:] if k in ("q", "k", "v", "g", "beta") else v) for k, v in inp.items()}
    b["state"] = sa
    ob, sb = gdn.kernel_fn(**b, mode="split")
    assert torch.equal(torch.cat([oa, ob], dim=1), out)
    assert torch.equal(sb, fs)


def test_gdn_deterministic(cuda_device):
    inp = gcfg.random_inputs(2, 700, seed=11, state_std=0.02)
    r = [gdn.kernel_fn(**inp) for _ in range(3)]
    for o, s in r[1:]:
        assert torch.equal(o, r[0][0]) and torch.equal(s, r[0][1])


def test_gdn_varlen_full_size(cuda_device, oracle_threads):
    """8 sequences, lengths ~U[1024, 32768], per-sequence initial state N(0, 0.02): the two
    shortest sequences against the oracle, every sequence against its own one-sequence run (all
    sequences against the oracle: tests/test_gdn_fullsize_gpu.py)."""
    lengths = gcfg.varlen_lengths(8, seed=0)
    inp = gcfg.random_inputs(1, 0, lengths=lengths, seed=0, state_std=0.02)
    out, fs = gdn.kernel_fn(**inp, mode="fused")
    gdn.check_device_status(cuda_device)
    cu = np.cumsum([0] + lengths)
    order = np.argsort(lengths)
    for n in range(8):
        a, b = int(cu[n]), int(cu[n + 1])
        one = {k: (v[:, a:b] if k in ("q", "k", "v", "g", "beta") else v) for k, v in inp.items() if k != "cu_seqlens"}
        one["state"] = inp["state"][n:n + 1]
        o1, s1 = gdn.kernel_fn(**one, mode="fused")  # the same kernel on one sequence: bit for bit
        assert torch.equal(o1, out[:, a:b]) and torch.equal(s1[0], fs[n]), n
        if n in order[:2]:
            o_ref, s_ref = _oracle({**one}, oracle_threads)
            np.testing.assert_allclose(_np(o1), o_ref, **OUT_TOL)
            np.testing.assert_allclose(_np(s1), s_ref, **STATE_TOL)


def _raw_qk_inputs(b, t, seed, scale=3.0, dtype=torch.bfloat16, hk=16, hv=32):
    """The random workload with q, k left unnormalised (N(0, scale^2))."""
    inp = gcfg.random_inputs(b, t, dtype=dtype, seed=seed, state_std=0.02, hk=hk, hv=hv)
    gen = torch.Generator().manual_seed(seed + 1)
    for n in ("q", "k"):
        inp[n] = (torch.randn(inp[n].shape, generator=gen) * scale).to(dtype).to(inp[n].device)
    return inp


def _normalised_for_oracle(inp):
    """The kernel's operands: q/|q|, k/|k| in fp32 then rounded to bf16, v rounded to bf16."""
    ref = dict(inp)
    for n in ("q", "k"):
        ref[n] = torch.from_numpy(oracle.l2norm_rows(_np(inp[n]))).to(torch.bfloat16)
    ref["v"] = inp["v"].to(torch.bfloat16)
    return ref


@pytest.mark.parametrize("b,t,dtype", [(1, 200, torch.bfloat16), (2, 65, torch.float32), (3, 1, torch.bfloat16)])
def test_gdn_qk_l2norm_matches_oracle(cuda_device, oracle_threads, b, t, dtype):
    """qk_l2norm=True on unnormalised q, k equals the recurrence on q/|q|, k/|k| (t=1 runs the decode kernel)."""
    inp = _raw_qk_inputs(b, t, seed=31 + t, dtype=dtype)
    out, fs = gdn.kernel_fn(**inp, qk_l2norm=True)
    o_ref, s_ref = _oracle(_normalised_for_oracle(inp), oracle_threads)
    np.testing.assert_allclose(_np(out), o_ref, **OUT_TOL)
    np.testing.assert_allclose(_np(fs), s_ref.reshape(fs.shape), **STATE_TOL)


def test_gdn_qk_l2norm_is_idempotent_on_normalised_inputs(cuda_device):
    inp = gcfg.random_inputs(1, 300, seed=8, state_std=0.02)
    a = gdn.kernel_fn(**inp)
    b = gdn.kernel_fn(**inp, qk_l2norm=True)
    np.testing.assert_allclose(_np(b[0]), _np(a[0]), **OUT_TOL)
    np.testing.assert_allclose(_np(b[1]), _np(a[1]), **STATE_TOL)


def test_l2norm_rows_kernel(cuda_device):
    gen = torch.Generator().manual_seed(2)
    for dtype in (torch.bfloat16, torch.float32):
        x = (torch.randn(5, 7, 16, 128, generator=gen) * 5.0).to(dtype).to(cuda_device)
        y = gdn.l2norm_rows(x)
        assert y.dtype == torch.bfloat16 and y.shape == x.shape
        ref = oracle.l2norm_rows(_np(x))
        np.testing.assert_allclose(_np(y), ref, atol=4e-3, rtol=8e-3)
    assert gdn.l2norm_rows(torch.zeros(0, 128, device=cuda_device)).shape == (0, 128)



@pytest.mark.parametrize("mode", ["auto", "split", "overlap"])
def test_gdn_checkpoints_match_prefix_oracle(cuda_device, oracle_threads, mode):
    """checkpoints[:, c] = the state after tokens [0, 64 (c+1)): the recurrence on that prefix."""
    inp = gcfg.random_inputs(2, 200, seed=21, state_std=0.02, hk=2, hv=4)
    out, fs, ck = gdn.kernel_fn(**inp, checkpoints=True, mode=mode)
    assert ck.shape == (2, 4, 4, 128, 128)
    ref_out, ref_fs = gdn.kernel_fn(**inp, mode=mode)
    assert torch.equal(out, ref_out) and torch.equal(fs, ref_fs)  # checkpoints change nothing else
    assert torch.equal(ck[:, -1], fs)
    for c in range(4):
        t_end = min(64 * (c + 1), 200)
        prefix = {n: (x[:, :t_end] if n in ("q", "k", "v", "g", "beta") else x) for n, x in inp.items()}
        _, s_ref = _oracle(prefix, oracle_threads)
        np.testing.assert_allclose(_np(ck[:, c]), s_ref, **STATE_TOL, err_msg=f"chunk {c}")


def test_gdn_checkpoints_varlen(cuda_device, oracle_threads):
    lengths = [1, 63, 64, 65, 200, 0, 129]
    inp = gcfg.random_inputs(1, 0, lengths=lengths, seed=6, state_std=0.02, hk=2, hv=4)
    out, fs, ck = gdn.kernel_fn(**inp, checkpoints=True)
    nch = [(n + 63) // 64 for n in lengths]
    assert ck.shape == (sum(nch), 4, 128, 128)
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + n)
    base = 0
    for s, n in enumerate(lengths):
        for c in range(nch[s]):
            t_end = cu[s] + min(64 * (c + 1), n)
            one = {"q": inp["q"][:, cu[s]:t_end], "k": inp["k"][:, cu[s]:t_end], "v": inp["v"][:, cu[s]:t_end],
                   "g": inp["g"][:, cu[s]:t_end], "beta": inp["beta"][:, cu[s]:t_end],
                   "state": inp["state"][s:s + 1], "scale": inp["scale"]}
            _, s_ref = _oracle(one, oracle_threads)
            np.testing.assert_allclose(_np(ck[base + c]), s_ref[0], **STATE_TOL, err_msg=f"seq {s} chunk {c}")
        if nch[s]:
            assert torch.equal(ck[base + nch[s] - 1], fs[s])
        base += nch[s]


def test_gdn_checkpoints_single_token_and_fused_refusal(cuda_device):
    inp = gcfg.random_inputs(3, 1, seed=2, state_std=0.02)
    out, fs, ck = gdn.kernel_fn(**inp, checkpoints=True)
    assert ck.shape == (3, 1, 32, 128, 128) and torch.equal(ck[:, 0], fs)
    with pytest.raises(ValueError):
        gdn.kernel_fn(**gcfg.random_inputs(1, 100, seed=2), checkpoints=True, mode="fused")


def _raw_gates(shape, hv, seed, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    a = (torch.randn(shape, generator=gen) * 2.0).to(dtype).cuda()
    b = (torch.randn(shape, generator=gen) * 2.0).to(dtype).cuda()
    a_log = torch.randn(hv, generator=gen) * 0.5
    dt_bias = torch.randn(hv, generator=gen) * 0.5
    return a, b, a_log, dt_bias


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gdn_gates_kernel_matches_oracle(cuda_device, dtype):
    a, b, a_log, dt_bias = _raw_gates((3, 70, 32), 32, seed=5, dtype=dtype)
    a[0, 0, 0] = 60.0  # the large-argument branch of softplus
    g, beta = gdn.gdn_gates(a, b, a_log, dt_bias)
    g_ref, b_ref = oracle.gdn_gates(_np(a), _np(b), a_log.numpy(), dt_bias.numpy())
    np.testing.assert_allclose(_np(g), g_ref, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(_np(beta), b_ref, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("t", [150, 1])
def test_gdn_with_raw_gates_matches_oracle(cuda_device, oracle_threads, t):
    """gates=(A_log, dt_bias): g, beta arguments are the raw projections (t=1 runs the decode kernel)."""
    inp = gcfg.random_inputs(2, t, seed=12 + t, state_std=0.02, hk=4, hv=8)
    a, b, a_log, dt_bias = _raw_gates(inp["g"].shape, 8, seed=13)
    out, fs = gdn.kernel_fn(**{**inp, "g": a, "beta": b}, gates=(a_log, dt_bias))
    g_ref, b_ref = oracle.gdn_gates(_np(a), _np(b), a_log.numpy(), dt_bias.numpy())
    o_ref, s_ref = _oracle({**inp, "g": torch.from_numpy(g_ref), "beta": torch.from_numpy(b_ref)}, oracle_threads)
    np.testing.assert_allclose(_np(out), o_ref, **OUT_TOL)
    np.testing.assert_allclose(_np(fs), s_ref.reshape(fs.shape), **STATE_TOL)


@pytest.mark.parametrize("mode", ["fused", "split", "overlap", "segmented"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gdn_gates_inside_the_kernels_equal_the_separate_pass(cuda_device, mode, dtype):
    """gates=(A_log, dt_bias): the preparation of each chunk computes g and beta from the raw
    projections with the separate pass's arithmetic, so the results are the same bits as running
    gdn_gates first and passing its g and beta."""
    inp = gcfg.random_inputs(1, 0, lengths=[70, 300, 1, 0, 129], seed=14, state_std=0.02, hk=2, hv=4)
    a, b, a_log, dt_bias = _raw_gates(inp["g"].shape, 4, seed=15, dtype=dtype)
    o1, s1 = gdn.kernel_fn(**{**inp, "g": a, "beta": b}, gates=(a_log, dt_bias), mode=mode, segment_chunks=2)
    g, beta = gdn.gdn_gates(a, b, a_log, dt_bias)
    o2, s2 = gdn.kernel_fn(**{**inp, "g": g, "beta": beta}, mode=mode, segment_chunks=2)
    gdn.check_device_status(cuda_device)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


@pytest.mark.parametrize("mode", ["fused", "split", "overlap", "segmented"])
def test_gdn_qk_l2norm_inside_the_kernels_equals_the_separate_pass(cuda_device, mode):
    """qk_l2norm=True on bf16 q, k: the rows are normalised as they are staged inside stage 1
    (with the separate pass's summation order), so the results are the same bits as running
    l2norm_rows first; with the gates computed inside stage 1 too."""
    inp = _raw_qk_inputs(2, 300, seed=61, hk=2, hv=4)
    o1, s1 = gdn.kernel_fn(**inp, qk_l2norm=True, mode=mode, segment_chunks=2)
    ref = {**inp, "q": gdn.l2norm_rows(inp["q"]), "k": gdn.l2norm_rows(inp["k"])}
    o2, s2 = gdn.kernel_fn(**ref, mode=mode, segment_chunks=2)
    gdn.check_device_status(cuda_device)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    a, b, a_log, dt_bias = _raw_gates(inp["g"].shape, 4, seed=62)
    o3, s3 = gdn.kernel_fn(**{**inp, "g": a, "beta": b}, gates=(a_log, dt_bias), qk_l2norm=True, mode=mode,
                           segment_chunks=2)
    g, beta = gdn.gdn_gates(a, b, a_log, dt_bias)
    o4, s4 = gdn.kernel_fn(**{**ref, "g": g, "beta": beta}, mode=mode, segment_chunks=2)
    gdn.check_device_status(cuda_device)
    assert torch.equal(o3, o4) and torch.equal(s3, s4)
