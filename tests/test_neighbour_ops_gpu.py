"""The harness's other registered row-wise ops on a B200 -- rms_norm, swiglu_input_quant and
qkv_part_rope through their plugin modules (``tokmix_rms_norm``, ``tokmix_swiglu_input_quant``,
``tokmix_qkv_part_rope`` in the C ABI) against the torch checkers the configs name: every config
size and dtype at the config's tolerance, then stricter properties (bytes that must be exact, one
output ulp elsewhere) and the edge shapes."""

import pytest
import torch

from kernel_opt_agent_b200 import qkv_part_rope as rope
from kernel_opt_agent_b200 import references
from kernel_opt_agent_b200 import rms_norm as rms
from kernel_opt_agent_b200 import swiglu_input_quant as swq
from kernel_opt_agent_b200.kernel_configs import KERNEL_CONFIGS

pytestmark = pytest.mark.gpu
MODULES = {"rms_norm": rms, "swiglu_input_quant": swq, "qkv_part_rope": rope}
# one rounding step of the output type (relative), with a floor for values near zero
ULP = {torch.bfloat16: dict(atol=1e-2, rtol=2 ** -7), torch.float16: dict(atol=1e-3, rtol=2 ** -10)}


def _config_cases(name):
    cfg = KERNEL_CONFIGS[name]
    return [(name, label, size, dt) for label, size in cfg["test_sizes"] + cfg["edge_sizes"]
            for dt in cfg["test_dtypes"]]


@pytest.mark.parametrize("name,label,size,dtype",
                         [c for n in MODULES for c in _config_cases(n)],
                         ids=lambda v: v if isinstance(v, str) else None)
def test_config_sizes_match_reference(cuda_device, name, label, size, dtype):
    cfg = KERNEL_CONFIGS[name]
    inp = cfg["input_generator"](size, dtype, str(cuda_device))
    got = MODULES[name].kernel_fn(**inp)
    ref = cfg["reference_fn"](inp)
    tol = cfg["tolerances"][dtype]
    got = got if isinstance(got, (tuple, list)) else [got]
    ref = ref if isinstance(ref, (tuple, list)) else [ref]
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        assert g.shape == r.shape and g.dtype == r.dtype
        torch.testing.assert_close(g.float(), r.float(), **tol)


# ------------------------------------------------------------------------------------ rms_norm
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 8), (3, 5, 136), (1023, 768), (2048, 5120), (7, 16384)])
def test_rms_norm_within_one_ulp(cuda_device, dtype, shape):
    gen = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=gen) * 3).to(dtype).to(cuda_device)
    w = torch.randn(shape[-1], generator=gen).to(dtype).to(cuda_device)
    out = rms.kernel_fn(x, w)
    ref = references.rms_norm_ref(x, w)
    assert out.shape == x.shape and out.dtype == dtype
    torch.testing.assert_close(out.float(), ref.float(), **ULP[dtype])


def test_rms_norm_zero_rows_and_eps(cuda_device):
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda_device)
    x[1] = 1.0
    w = torch.full((64,), 2.0, dtype=torch.bfloat16, device=cuda_device)
    out = rms.kernel_fn(x, w, eps=1e-6)
    assert torch.equal(out[0], torch.zeros_like(out[0]))          # 0 / sqrt(eps) = 0
    torch.testing.assert_close(out[1].float(), torch.full((64,), 2.0, device=cuda_device), atol=1e-2, rtol=0)
    assert rms.kernel_fn(torch.empty(0, 64, dtype=torch.bfloat16, device=cuda_device), w).shape == (0, 64)


def test_rms_norm_rejects_bad_inputs(cuda_device):
    x = torch.randn(4, 64, device=cuda_device)
    with pytest.raises(ValueError):
        rms.kernel_fn(x, torch.ones(64, device=cuda_device))          # fp32
    xb = x.to(torch.bfloat16)
    with pytest.raises(ValueError):
        rms.kernel_fn(xb, torch.ones(32, dtype=torch.bfloat16, device=cuda_device))
    with pytest.raises(ValueError):
        rms.kernel_fn(xb[:, :60], torch.ones(60, dtype=torch.bfloat16, device=cuda_device))  # N % 8


# ---------------------------------------------------------------------------- swiglu_input_quant
@pytest.mark.parametrize("m,n", [(1, 128), (5, 256), (256, 1024), (1000, 3584), (4096, 7168)])
def test_swiglu_quant_bytes_exact(cuda_device, m, n):
    gen = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, 2 * n, generator=gen).to(torch.bfloat16).to(cuda_device)
    out, x_fp8, x_scale = swq.kernel_fn(x)
    r_out, r_fp8, r_scale = references.swiglu_input_quant_ref(x)
    assert torch.equal(x_scale, r_scale)                                       # same rounding of amax / 448
    assert torch.equal(x_fp8.view(torch.uint8), r_fp8.view(torch.uint8))       # same bf16 product, same rounding
    torch.testing.assert_close(out.float(), r_out.float(), **ULP[torch.bfloat16])


def test_swiglu_quant_zero_and_extreme_blocks(cuda_device):
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(6, 512, generator=gen)
    x[0] = 0.0                      # amax clamps to eps; quantised block is zero
    x[1, :128] = 3.0e38             # near the bf16 maximum
    x[2, 128:256] = 1e-30           # tiny magnitudes
    x[3, 5] = -448.0                # the e4m3 maximum lands exactly
    x = x.to(torch.bfloat16).to(cuda_device)
    out, x_fp8, x_scale = swq.kernel_fn(x)
    r_out, r_fp8, r_scale = references.swiglu_input_quant_ref(x)
    assert torch.equal(x_scale, r_scale)
    assert torch.equal(x_fp8.view(torch.uint8), r_fp8.view(torch.uint8))
    assert torch.equal(x_fp8[0].view(torch.uint8), torch.zeros(512, dtype=torch.uint8, device=cuda_device))
    finite = torch.isfinite(r_out.float())
    torch.testing.assert_close(out.float()[finite], r_out.float()[finite], **ULP[torch.bfloat16])


def test_swiglu_quant_rejects_bad_inputs(cuda_device):
    with pytest.raises(ValueError):
        swq.kernel_fn(torch.randn(4, 192, dtype=torch.bfloat16, device=cuda_device))   # 2N % 256
    with pytest.raises(ValueError):
        swq.kernel_fn(torch.randn(4, 256, device=cuda_device))                          # fp32
    empty = swq.kernel_fn(torch.empty(0, 256, dtype=torch.bfloat16, device=cuda_device))
    assert [t.shape for t in empty] == [(0, 128), (0, 256), (2, 0)]


# --------------------------------------------------------------------------------- qkv_part_rope
@pytest.mark.parametrize("b,s,qh,kvh,d,nope,neg", [
    (1, 2048, 10, 1, 256, 192, False),
    (2, 333, 10, 1, 256, 192, True),
    (3, 17, 4, 2, 128, 64, False),
    (1, 5, 8, 0, 64, 0, False),          # full rotation, no key heads
    (2, 9, 2, 2, 96, 96, False),         # nothing rotated: a copy
    (2, 7, 3, 1, 320, 256, False),       # head_dim above 256: the per-row kernel
    (1, 11, 5, 3, 64, 40, True),         # rope half of 12 columns: the per-row kernel
])
def test_qkv_rope_matches_reference(cuda_device, b, s, qh, kvh, d, nope, neg):
    inp = rope.get_inputs(batch=b, seq_len=s, q_heads=qh, kv_heads=kvh, head_dim=d, nope_dim=nope,
                          seed=b * s + d, device=str(cuda_device))
    out = rope.kernel_fn(**inp, negative_sin=neg)
    ref = references.qkv_part_rope_ref(**inp, negative_sin=neg)
    assert out.shape == ref.shape and out.dtype == torch.bfloat16
    nrot = qh + kvh
    assert torch.equal(out[:, :, nrot:], inp["qkv"][:, :, nrot:])           # value heads pass through
    assert torch.equal(out[..., :nope], inp["qkv"][..., :nope])             # nope columns pass through
    assert torch.equal(out, ref)    # products and sums rounded one by one, as the checker's tensor ops


def test_qkv_rope_three_dim_input(cuda_device):
    inp = rope.get_inputs(batch=1, seq_len=64, device=str(cuda_device))
    inp["qkv"] = inp["qkv"][0]
    out = rope.kernel_fn(**inp)
    ref = references.qkv_part_rope_ref(**inp)
    assert out.shape == ref.shape == (1, 64, 12, 256)
    assert torch.equal(out, ref)


def test_qkv_rope_rejects_bad_inputs(cuda_device):
    inp = rope.get_inputs(batch=1, seq_len=16, device=str(cuda_device))
    with pytest.raises(ValueError):
        rope.kernel_fn(**{**inp, "cos": inp["cos"][:8]})
    with pytest.raises(ValueError):
        rope.kernel_fn(**{**inp, "q_heads": 12})
    with pytest.raises(ValueError):
        rope.kernel_fn(**{**inp, "qkv": inp["qkv"].float()})
