"""The oracle against the reference's own outputs and against independent restatements (CPU)."""

import json
import math
import pathlib

import numpy as np
import pytest
import torch

import oracle
from tests.golden import make_golden as golden

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name", sorted(golden.FA2_CASES))
def test_fa2_oracle_matches_sdpa_golden(name):
    case = golden.FA2_CASES[name]
    q, k, v = golden.fa2_inputs(case)
    if case["layout"] == "bshd":
        q, k, v = (x.transpose(1, 2) for x in (q, k, v))
    out = oracle.fa2_attention(q.numpy(), k.numpy(), v.numpy(), causal=case["causal"])
    if case["layout"] == "bshd":
        out = out.transpose(0, 2, 1, 3)
    ref = np.load(GOLDEN / f"{name}.npz")["out_fp32"]
    np.testing.assert_allclose(out, ref, atol=2e-6, rtol=2e-5)
    # the reference itself runs SDPA in bf16: the fp32 oracle is within bf16 rounding of it
    np.testing.assert_allclose(out, np.load(GOLDEN / f"{name}.npz")["out_sdpa_bf16"], atol=2e-2, rtol=2e-2)


def test_fa2_oracle_matches_live_sdpa_gqa_noncausal():
    import torch.nn.functional as F

    gen = torch.Generator().manual_seed(5)
    q = torch.randn(2, 6, 70, 64, generator=gen)
    k = torch.randn(2, 3, 90, 64, generator=gen)
    v = torch.randn(2, 3, 90, 64, generator=gen)
    for causal in (False, True):
        ref = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=0.3, enable_gqa=True).numpy()
        out = oracle.fa2_attention(q.numpy(), k.numpy(), v.numpy(), causal=causal, sm_scale=0.3)
        np.testing.assert_allclose(out, ref, atol=3e-6, rtol=3e-5)


def _gdn_case(b, t, hk, hv, seed, state=True, gscale=1.0):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(b, t, hk, 128, generator=gen)
    k = torch.randn(b, t, hk, 128, generator=gen)
    q = q / q.norm(dim=-1, keepdim=True)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(b, t, hv, 128, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(b, t, hv, generator=gen)) * gscale
    beta = torch.sigmoid(torch.randn(b, t, hv, generator=gen))
    st = torch.randn(b, hv, 128, 128, generator=gen) * 0.02 if state else None
    return [x.numpy() if x is not None else None for x in (q, k, v, g, beta, st)]


def test_gdn_c_oracle_matches_numpy_transcription():
    q, k, v, g, beta, st = _gdn_case(2, 37, 2, 4, seed=1)
    o1, s1 = oracle.gdn_recurrent(q, k, v, g, beta, st)
    o2, s2 = oracle.gdn_recurrent_numpy(q, k, v, g, beta, st)
    np.testing.assert_allclose(o1, o2, atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(s1, s2, atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("gscale", [1.0, 0.02])
def test_gdn_recurrence_matches_chunked_form(gscale):
    """The chunked (UT/WY) restatement, a different algorithm, agrees with the recurrence."""
    q, k, v, g, beta, st = _gdn_case(1, 150, 2, 4, seed=2, gscale=gscale)
    o1, s1 = oracle.gdn_recurrent(q, k, v, g, beta, st)
    o2, s2 = oracle.gdn_chunked_numpy(q, k, v, g, beta, st, chunk=64)
    np.testing.assert_allclose(o1, o2, atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(s1, s2, atol=2e-5, rtol=1e-4)


def test_gdn_varlen_equals_per_sequence():
    q, k, v, g, beta, _ = _gdn_case(1, 100, 2, 4, seed=3, state=False)
    lens = [0, 30, 1, 69]
    cu = np.cumsum([0] + lens)
    st = np.random.default_rng(0).standard_normal((4, 4, 128, 128)).astype(np.float32) * 0.02
    o, s = oracle.gdn_recurrent(q, k, v, g, beta, st, cu_seqlens=cu)
    for n in range(4):
        a, b = cu[n], cu[n + 1]
        o1, s1 = oracle.gdn_recurrent(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b], st[n:n + 1])
        np.testing.assert_array_equal(o[:, a:b], o1)
        np.testing.assert_array_equal(s[n], s1[0])


def test_gdn_state_continuation():
    q, k, v, g, beta, st = _gdn_case(1, 90, 1, 2, seed=4)
    o, s = oracle.gdn_recurrent(q, k, v, g, beta, st)
    oa, sa = oracle.gdn_recurrent(q[:, :41], k[:, :41], v[:, :41], g[:, :41], beta[:, :41], st)
    ob, sb = oracle.gdn_recurrent(q[:, 41:], k[:, 41:], v[:, 41:], g[:, 41:], beta[:, 41:], sa)
    np.testing.assert_array_equal(np.concatenate([oa, ob], axis=1), o)
    np.testing.assert_array_equal(sb, s)


def _gdn_golden_available():
    return (GOLDEN / "gdn_golden_meta.json").exists()


@pytest.mark.skipif(not _gdn_golden_available(), reason="GDN golden vectors not generated yet")
@pytest.mark.parametrize("name", sorted(golden.GDN_CASES))
def test_gdn_oracle_matches_reference_kernel_golden(name):
    """Pin: outputs of the reference's own fp32 CUDA kernel (run on a B200)."""
    meta = json.loads((GOLDEN / "gdn_golden_meta.json").read_text())
    q, k, v, g, beta, st = (x.numpy() for x in golden.gdn_inputs(golden.GDN_CASES[name]))
    o, s = oracle.gdn_recurrent(q, k, v, g, beta, st)
    ref = np.load(GOLDEN / f"{name}.npz")
    np.testing.assert_allclose(o[:, :, meta["out_heads"]], ref["out"], atol=1e-6, rtol=1e-4)
    np.testing.assert_allclose(s[:, meta["state_heads"]], ref["final_state"], atol=1e-6, rtol=1e-4)


def test_gdn_strong_negative_gate_is_finite():
    q, k, v, g, beta, st = _gdn_case(1, 64, 1, 2, seed=6)
    g = np.random.default_rng(1).uniform(-25, -8, g.shape).astype(np.float32)
    o, s = oracle.gdn_recurrent(q, k, v, g, beta, st)
    assert np.isfinite(o).all() and np.isfinite(s).all()
    o2, s2 = oracle.gdn_chunked_numpy(q, k, v, g, beta, st)
    np.testing.assert_allclose(o, o2, atol=1e-5, rtol=1e-4)


def test_l2norm_rows_oracle_unit_rows():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((6, 128)).astype(np.float32) * 4
    y = oracle.l2norm_rows(x)
    np.testing.assert_allclose(np.linalg.norm(y, axis=-1), 1.0, rtol=1e-5)
    np.testing.assert_allclose(oracle.l2norm_rows(np.zeros((2, 128), np.float32)), 0.0)


def test_gdn_gates_oracle_formula():
    a = np.array([[0.0, 30.0, -30.0]], np.float32)
    b = np.array([[0.0, 5.0, -5.0]], np.float32)
    g, beta = oracle.gdn_gates(a, b, np.zeros(3, np.float32), np.zeros(3, np.float32))
    np.testing.assert_allclose(g, [[-np.log(2.0), -30.0, -np.log1p(np.exp(-30.0))]], rtol=1e-6)
    np.testing.assert_allclose(beta, [[0.5, 1 / (1 + np.exp(-5.0)), 1 / (1 + np.exp(5.0))]], rtol=1e-6)
