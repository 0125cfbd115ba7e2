"""The allocation-free GDN entry point, tokmix_gdn_prefill_noalloc, called through the C ABI.

It serves callers that cannot allocate device memory while running an op -- graph executors
that plan every buffer ahead of time, or C / FFI code without a device allocator.  Those callers
pass only their inputs and outputs; the token offsets and the status word the kernel needs live
in a small library-owned device array instead.  The test (which itself may allocate) checks that
two calls in a row, with different batch sizes so the shared array is rewritten in between,
give bit for bit what the regular entry point gives (both run the same one-CTA-per-unit
kernel), and that the library's status word, used when the caller passes none, reads zero
afterwards.  This file is named to run last.
"""

import ctypes

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


def _library_status(clear=True):
    word = ctypes.c_uint32(0xFFFFFFFF)
    _lib.check(_lib.load().tokmix_gdn_noalloc_status(ctypes.addressof(word), 1 if clear else 0),
               "tokmix_gdn_noalloc_status")
    return word.value


def test_noalloc_matches_regular_entry_point_twice(cuda_device):
    cases = [gcfg.random_inputs(3, 200, seed=21, state_std=0.02, hk=4, hv=8),
             gcfg.random_inputs(2, 129, seed=22, state_std=0.02)]
    word = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for i, inp in enumerate(cases):
        ref_out, ref_state = gdn.kernel_fn(**inp, mode="fused")
        out, final = _noalloc(inp, status=None if i == 0 else word)
        torch.cuda.synchronize()
        if i == 0:  # the kernels' status bits went to the library's own word
            assert _library_status() == 0
        assert torch.equal(out, ref_out) and torch.equal(final, ref_state)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref_out.float().cpu().numpy(), **OUT_TOL)
        np.testing.assert_allclose(final.cpu().numpy(), ref_state.cpu().numpy(), **STATE_TOL)
    assert int(word.item()) == 0


def test_noalloc_rejects_oversized_batch(cuda_device):
    lib = _lib.load()
    p = 16
    rc = lib.tokmix_gdn_prefill_noalloc(p, p, p, p, p, None, p, p, 4096, 64, 16, 32, 128, 128, 0.088, 0, None, None)
    assert rc == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "4095" in _lib.last_error()


def test_noalloc_rejects_bad_arguments_before_touching_its_array(cuda_device):
    """A rejected call enqueues nothing: the shared offsets of an earlier call stay valid.  The
    rejected calls get buffers large enough for the shapes they name, so that nothing they could
    run reads or writes outside them."""
    inp = gcfg.random_inputs(2, 129, seed=23, state_std=0.02, hk=4, hv=8)
    ref_out, ref_state = gdn.kernel_fn(**inp, mode="fused")
    out, final = _noalloc(inp)
    bad = gcfg.random_inputs(7, 64, seed=24, hk=4, hv=8)
    pad = torch.zeros(bad["q"].numel() + 64, dtype=torch.bfloat16, device=cuda_device)
    bad_out = torch.empty_like(bad["v"])
    bad_final = torch.empty((7, 8, 128, 128), dtype=torch.float32, device=cuda_device)
    args = [bad[x].data_ptr() for x in ("q", "k", "v", "g", "beta")] + [None, bad_out.data_ptr(),
                                                                         bad_final.data_ptr()]
    lib = _lib.load()
    misaligned = list(args)
    misaligned[0] = pad.data_ptr() + 2  # q not 16-byte aligned
    rc = lib.tokmix_gdn_prefill_noalloc(*misaligned, 7, 64, 4, 8, 128, 128, 0.088, 0, None, None)
    assert rc == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "aligned" in _lib.last_error()
    rc = lib.tokmix_gdn_prefill_noalloc(*args, 7, 64, 4, 6, 128, 128, 0.088, 0, None, None)
    assert rc == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "multiple" in _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(final, ref_state)
