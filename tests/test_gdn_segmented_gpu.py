"""The segmented GDN schedule on a B200 (tokmix_gdn_prefill_segmented, through the plugin
module): long sequences cut into segments whose chains run side by side -- a zero-start chain
and a transition chain (identity start, zero values) for each later segment -- then joined by the
fp32 combine of the entry states and the tensor-core correction of the outputs.  Checked against
the fp32 recurrence oracle at the GPU tests' tolerances, with segment lengths forced small so
that sequences are cut into many segments, including 1-token and 1-chunk segments."""

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=2e-2, rtol=2e-2)
STATE_TOL = dict(atol=1e-4, rtol=1e-3)


def _np(x):
    return None if x is None else x.float().cpu().numpy()


def _oracle(inp, threads):
    return oracle.gdn_recurrent(_np(inp["q"]), _np(inp["k"]), _np(inp["v"]), _np(inp["g"]), _np(inp["beta"]),
                                _np(inp.get("state")), inp.get("scale"), cu_seqlens=_np(inp.get("cu_seqlens")),
                                nthreads=threads)


def _check(inp, threads, seg=None):
    out, fs = gdn.kernel_fn(**inp, mode="segmented", segment_chunks=seg)
    gdn.check_device_status(out.device)
    o_ref, s_ref = _oracle(inp, threads)
    assert np.isfinite(_np(out)).all() and np.isfinite(_np(fs)).all()
    np.testing.assert_allclose(_np(out), o_ref, **OUT_TOL)
    np.testing.assert_allclose(_np(fs), s_ref.reshape(fs.shape), **STATE_TOL)
    return out, fs


@pytest.mark.parametrize("b,t,seg,state_std", [
    (1, 640, 3, 0.0),     # 10 chunks -> segments of 3, 3, 2, 2
    (2, 300, 2, 0.02),    # 5 chunks (last one 44 tokens) -> 2, 2, 1
    (1, 257, 2, 0.02),    # the last segment is one chunk of one token
    (3, 129, 1, 0.02),    # every chunk its own segment
    (1, 2048, 5, 0.02),   # 32 chunks -> 7 segments
])
def test_segmented_matches_oracle(cuda_device, oracle_threads, b, t, seg, state_std):
    inp = gcfg.random_inputs(b, t, seed=t + seg, state_std=state_std, hk=2, hv=4)
    _check(inp, oracle_threads, seg)


def test_segmented_varlen_mixed_lengths(cuda_device, oracle_threads):
    """Whole sequences (empty, 1 token, short) next to cut ones in one call."""
    inp = gcfg.random_inputs(1, 0, lengths=[1, 63, 64, 65, 700, 0, 1000, 129], seed=41, state_std=0.02, hk=2, hv=4)
    _check(inp, oracle_threads, seg=4)


def test_segmented_strong_and_weak_decay(cuda_device, oracle_threads):
    inp = gcfg.random_inputs(1, 1024, seed=42, state_std=0.02, hk=2, hv=4)
    gen = torch.Generator().manual_seed(43)
    inp["g"] = (torch.rand(inp["g"].shape, generator=gen) * 17.0 - 25.0).cuda()
    _check(inp, oracle_threads, seg=3)
    weak = gcfg.random_inputs(1, 4096, seed=44, state_std=0.02, hk=2, hv=4)
    weak["g"] = torch.full_like(weak["g"], -0.002)
    _check(weak, oracle_threads, seg=8)


def test_segmented_config1_full(cuda_device, oracle_threads):
    """B=1, T=2048, Hk=16, Hv=32 with the planner's own segment length."""
    inp = gcfg.random_inputs(1, 2048, seed=0)
    _check(inp, oracle_threads)


def test_segmented_is_deterministic_and_close_to_unsegmented(cuda_device):
    inp = gcfg.random_inputs(2, 1500, seed=45, state_std=0.02, hk=4, hv=8)
    runs = [gdn.kernel_fn(**inp, mode="segmented", segment_chunks=6) for _ in range(3)]
    for o, s in runs[1:]:
        assert torch.equal(o, runs[0][0]) and torch.equal(s, runs[0][1])
    o_ref, s_ref = gdn.kernel_fn(**inp, mode="split")
    np.testing.assert_allclose(_np(runs[0][0]), _np(o_ref), **OUT_TOL)
    np.testing.assert_allclose(_np(runs[0][1]), _np(s_ref), **STATE_TOL)


def test_segmented_varlen_workload_head_slice(cuda_device, oracle_threads):
    """The 8-sequence varlen workload restricted to 2 key heads (4 value heads: one GPU's share of
    8), as the schedule is used there: the planner cuts the sequences, every token checked."""
    lengths = gcfg.varlen_lengths(8, seed=0)
    inp = gcfg.random_inputs(1, 0, lengths=lengths, seed=0, state_std=0.02, hk=2, hv=4)
    assert gdn.schedule(inp["q"], inp["v"], inp["cu_seqlens"], mode="segmented") == "segmented"
    _check(inp, oracle_threads)
