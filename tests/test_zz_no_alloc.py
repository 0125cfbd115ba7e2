"""The allocation-free GDN entry point, tokmix_gdn_prefill_noalloc, called through the C ABI.

It serves callers that cannot allocate device memory while running an op -- graph executors
that plan every buffer ahead of time, or C / FFI code without a device allocator.  Those callers
pass only their inputs and outputs; the token offsets and the status word the kernel needs live
in a small library-owned device array instead.  The test (which itself may allocate) checks that
two calls in a row, with different batch sizes so the shared array is rewritten in between,
match the regular entry point within the GPU tests' tolerances.  This file is named to run last.
"""

import numpy as np
import pytest
import torch

from kernel_opt_agent_b200 import _lib
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=2e-2, rtol=2e-2)
STATE_TOL = dict(atol=1e-4, rtol=1e-3)


def _noalloc(inp, status=None):
    q, k, v, g, beta, st = (inp[x] for x in ("q", "k", "v", "g", "beta", "state"))
    B, T, hk = q.shape[0], q.shape[1], q.shape[2]
    hv = v.shape[2]
    out = torch.empty_like(v)
    final = torch.empty((B, hv, 128, 128), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    rc = lib.tokmix_gdn_prefill_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), st.data_ptr(), out.data_ptr(),
        final.data_ptr(), B, T, hk, hv, 128, 128, float(inp["scale"]), _lib.DTYPE_BF16,
        status.data_ptr() if status is not None else None, torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(rc, "tokmix_gdn_prefill_noalloc")
    return out, final


def test_noalloc_matches_regular_entry_point_twice(cuda_device):
    cases = [gcfg.random_inputs(3, 200, seed=21, state_std=0.02, hk=4, hv=8),
             gcfg.random_inputs(2, 129, seed=22, state_std=0.02)]
    word = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for i, inp in enumerate(cases):
        ref_out, ref_state = gdn.kernel_fn(**inp)
        out, final = _noalloc(inp, status=None if i == 0 else word)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref_out.float().cpu().numpy(), **OUT_TOL)
        np.testing.assert_allclose(final.cpu().numpy(), ref_state.cpu().numpy(), **STATE_TOL)
    assert int(word.item()) == 0


def test_noalloc_rejects_oversized_batch(cuda_device):
    lib = _lib.load()
    p = 16
    rc = lib.tokmix_gdn_prefill_noalloc(p, p, p, p, p, None, p, p, 4096, 64, 16, 32, 128, 128, 0.088, 0, None, None)
    assert rc == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "4095" in _lib.last_error()
