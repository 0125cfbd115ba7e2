"""The bounded-wait path on a B200: a wait that runs out sets its status bit, ends the kernel,
and surfaces on the host as TokmixDeviceError; the GPU stays usable afterwards.

The waits are the library's own (mbar_wait / wait_flag in csrc/sm100.cuh), run by
tokmix_selftest_wait_timeout on events that nothing satisfies, with a 1 ms limit; nothing is in
flight in that kernel (no TMA copy, MMA or TMEM), so the run ends cleanly.  The reference puts
its timeout around whole runs on the host (tools/bench.py:138-169).
"""

import time

import numpy as np
import pytest
import torch

import oracle
from kernel_opt_agent_b200 import _lib
from kernel_opt_agent_b200 import flash_attention_2 as fa2
from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn
from kernel_opt_agent_b200.kernel_configs import qwen35moe_gdn_prefill as gcfg

pytestmark = pytest.mark.gpu
LIMIT_NS = 1_000_000  # 1 ms


def _run(which, flag_value=0):
    dev = torch.device("cuda", 0)
    word = torch.zeros(1, dtype=torch.int32, device=dev)
    flag = torch.full((1,), flag_value, dtype=torch.int32, device=dev)
    result = torch.full((2,), -1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = _lib.load().tokmix_selftest_wait_timeout(which, LIMIT_NS, flag.data_ptr(), result.data_ptr(),
                                                  word.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc, "tokmix_selftest_wait_timeout")
    torch.cuda.synchronize()
    return word, result.cpu().tolist(), time.perf_counter() - t0


@pytest.mark.parametrize("which,bit", [(0, 0x1), (1, 0x4), (2, 0x4)])
def test_wait_that_runs_out_sets_its_bit_and_ends(cuda_device, which, bit):
    word, result, elapsed = _run(which)
    # both warps gave up: the first on its 1 ms limit, the second (2 s limit) on the CTA abort flag
    assert result == [0, 0]
    assert int(word.item()) == bit
    assert elapsed < 1.0
    with pytest.raises(_lib.TokmixDeviceError):
        _lib.raise_on_device_status(word, "selftest")
    assert int(word.item()) == 0  # cleared by the raise


def test_satisfied_flag_wait_reports_nothing(cuda_device):
    word, result, _ = _run(2, flag_value=1)
    assert result == [1, 1] and int(word.item()) == 0


def test_asynchronous_status_check_raises_at_the_next_call(cuda_device):
    """A bit in the plugin modules' status word surfaces without an explicit synchronisation: the
    copy queued behind a launch is read by a later call."""
    if _lib._STATUS_MODE != "async":
        pytest.skip("TOKMIX_CHECK_STATUS selects another mode")
    inp = gcfg.random_inputs(1, 70, seed=3, hk=2, hv=4)
    gdn.kernel_fn(**inp)
    gdn.check_device_status(cuda_device)
    word = _lib.status_word(cuda_device)
    word.fill_(0x4)  # as a kernel's timed-out hand-off would leave it
    with pytest.raises(_lib.TokmixDeviceError):
        for _ in range(50):
            gdn.kernel_fn(**inp)
            time.sleep(0.01)
    assert int(word.item()) == 0


def test_gpu_still_works_after_timeouts(cuda_device, oracle_threads):
    for which in (0, 1, 2):
        _run(which)
    inp = fa2.get_inputs(1, 2, 130, 128, seed=1, device="cuda")
    out = fa2.kernel_fn(**inp)
    fa2.check_device_status(cuda_device)
    ref = oracle.fa2_attention(*(inp[x].float().cpu().numpy() for x in ("q", "k", "v")), causal=True)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=2e-2)
    g_in = gcfg.random_inputs(1, 130, seed=2, state_std=0.02, hk=2, hv=4)
    o, s = gdn.kernel_fn(**g_in)
    gdn.check_device_status(cuda_device)
    ro, rs = oracle.gdn_recurrent(*(g_in[x].float().cpu().numpy() for x in ("q", "k", "v", "g", "beta")),
                                  g_in["state"].cpu().numpy(), g_in["scale"], nthreads=oracle_threads)
    np.testing.assert_allclose(o.float().cpu().numpy(), ro, atol=2e-2, rtol=2e-2)
    np.testing.assert_allclose(s.cpu().numpy(), rs, atol=1e-4, rtol=1e-3)


def test_selftest_rejects_bad_arguments():
    lib = _lib.load()
    assert lib.tokmix_selftest_wait_timeout(3, LIMIT_NS, None, None, 16, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_selftest_wait_timeout(0, 10, None, None, 16, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_selftest_wait_timeout(0, 2_000_000_000, None, None, 16, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_selftest_wait_timeout(2, LIMIT_NS, None, None, 16, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT


def _prefill_args(inp):
    q, k, v, g, beta, st = (inp[x] for x in ("q", "k", "v", "g", "beta", "state"))
    out = torch.empty_like(v)
    final = torch.empty(st.shape, dtype=torch.float32, device=q.device)
    return q, k, v, g, beta, st, out, final


def test_inconsistent_device_offsets_set_bad_args_bit(cuda_device):
    """Token offsets and chunk bases live on the device, where the host does not check them: a
    sequence whose offsets run backwards (one-CTA-per-unit kernel) or whose chunk base points
    past the workspace (record-fed chain) sets TOKMIX_DEV_BAD_ARGS and is skipped, while the
    consistent sequence of the same call is still computed."""
    lib = _lib.load()
    inp = gcfg.random_inputs(1, 128, seed=4, state_std=0.02, hk=2, hv=4)
    inp["state"] = torch.cat([inp["state"], inp["state"]])  # two sequences
    q, k, v, g, beta, st, out, final = _prefill_args(inp)
    ref_o, ref_s = gdn.kernel_fn(q[:, :64], k[:, :64], v[:, :64], g[:, :64], beta[:, :64], inp["state"][:1],
                                 inp["scale"], mode="fused")
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    # fused kernel: sequence 1 = tokens [64, 32): backwards
    word = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    cu = torch.tensor([0, 64, 32], dtype=torch.int32, device=cuda_device)
    rc = lib.tokmix_gdn_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), st.data_ptr(),
                                out.data_ptr(), final.data_ptr(), cu.data_ptr(), None, 2, 128, 2, 4, 128, 128,
                                float(inp["scale"]), _lib.DTYPE_BF16, None, word.data_ptr(), stream)
    _lib.check(rc, "tokmix_gdn_prefill")
    torch.cuda.synchronize()
    assert int(word.item()) == 0x8
    assert torch.equal(out[:, :64], ref_o) and torch.equal(final[:1], ref_s)
    # record-fed chain: sequence 1's chunk base lies past the two records of the workspace
    word.zero_()
    cu = torch.tensor([0, 64, 128], dtype=torch.int32, device=cuda_device)
    cb = torch.tensor([0, 5, 6], dtype=torch.int32, device=cuda_device)
    nbytes = int(lib.tokmix_gdn_split_workspace_bytes(2, 4))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    out.zero_()
    rc = lib.tokmix_gdn_prefill_split(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(),
                                      st.data_ptr(), out.data_ptr(), final.data_ptr(), None, cu.data_ptr(), cb.data_ptr(),
                                      None, 2, 128, 2, 2, 4, 128, 128, float(inp["scale"]), _lib.DTYPE_BF16, None,
                                      ws.data_ptr(), nbytes, word.data_ptr(), stream)
    _lib.check(rc, "tokmix_gdn_prefill_split")
    torch.cuda.synchronize()
    assert int(word.item()) == 0x8
    assert torch.equal(out[:, :64], ref_o) and torch.equal(final[:1], ref_s)
