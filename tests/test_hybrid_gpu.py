"""The hybrid prefill sweep's shapes on a B200 against the oracle: FA2 causal GQA Hq=16 Hkv=2
D=256 at sequence lengths 16384 and 65536 (sampled query rows against the fp32 softmax), and GDN
prefill Hk=16 Hv=32 at batch 16 x 4096 tokens (512 (sequence, head) units: more than the GPU has
SMs, so the one-CTA-per-unit schedule in several waves) and at 5 x 65536 tokens (160 units of
1024 chunks each), every head and every token compared with the fp32 recurrence."""

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import flash_attention_2 as fa2
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-2, rtol=2e-2)
STATE_TOL = dict(atol=1e-4, rtol=1e-3)


def _np(x):
    return x.float().cpu().numpy()


@pytest.mark.parametrize("s", [16384, 65536])
def test_hybrid_attention_long_sequences_sampled_rows(cuda_device, s):
    inp = fa2.get_inputs(1, 16, s, 256, seed=s, head_num_kv=2)
    out = fa2.kernel_fn(**inp)
    fa2.check_device_status(cuda_device)
    rng = np.random.default_rng(s)
    rows = [(0, 0), (15, s - 1), (7, 127), (8, 128), (3, s // 2 - 1), (12, s // 2), (1, s - 129)]
    rows += [(int(rng.integers(16)), int(rng.integers(s))) for _ in range(24)]
    for h, i in rows:
        q = inp["q"][0, h, i].float().cpu().numpy()
        kk = inp["k"][0, h // 8, : i + 1].float().cpu().numpy()
        vv = inp["v"][0, h // 8, : i + 1].float().cpu().numpy()
        sc = kk @ q * inp["sm_scale"]
        p = np.exp(sc - sc.max())
        ref = (p @ vv) / p.sum()
        np.testing.assert_allclose(out[0, h, i].float().cpu().numpy(), ref, **TOL, err_msg=str((h, i)))


_ORACLE_CACHE = {}


@pytest.mark.parametrize("mode", ["auto", "fused"])
@pytest.mark.parametrize("b,t", [(16, 4096), (5, 65536)])
def test_hybrid_gdn_matches_oracle(cuda_device, oracle_threads, b, t, mode):
    """More units than SMs: the one-CTA-per-unit kernel in waves, and the schedule "auto" picks
    (the record-fed chains run longest first when that is predicted faster)."""
    inp = gcfg.random_inputs(b, t, seed=b * t, state_std=0.02)
    out, fs = gdn.kernel_fn(**inp, mode=mode)
    gdn.check_device_status(cuda_device)
    if (b, t) not in _ORACLE_CACHE:
        _ORACLE_CACHE[(b, t)] = oracle.gdn_recurrent(*(_np(inp[x]) for x in ("q", "k", "v", "g", "beta")),
                                                     _np(inp["state"]), inp["scale"], nthreads=oracle_threads)
    o_ref, s_ref = _ORACLE_CACHE[(b, t)]
    np.testing.assert_allclose(_np(out), o_ref, **TOL, err_msg=gdn.schedule(inp["q"], inp["v"], mode=mode))
    np.testing.assert_allclose(_np(fs), s_ref, **STATE_TOL)
