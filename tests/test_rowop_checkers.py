"""The repository's row-op checkers (kernel_opt_agent_b200/references/{rms_norm,swiglu_input_quant,
qkv_part_rope}.py), which the GPU tests hold the CUDA kernels to bit for bit, pinned against the
reference's own checkers (references/*.py): on the CPU, every output bit equal to the reference
checker's output stored in tests/golden/rowop_*.npz (made by tests/golden/make_golden.py
--rowops from the reference checkout), and, where the checkout is present, on further live
cases."""

import pathlib

import numpy as np
import pytest
import torch

from kernel_opt_agent_b200 import references as ours
from tests.golden import make_golden as golden

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
REFERENCE = pathlib.Path("/root/reference")
OURS = {"rms_norm": ours.rms_norm_ref, "swiglu_input_quant": ours.swiglu_input_quant_ref,
        "qkv_part_rope": ours.qkv_part_rope_ref}


def _outputs(fn, inputs):
    res = fn(**inputs)
    return [golden.raw(t) for t in (res if isinstance(res, tuple) else (res,))]


@pytest.mark.parametrize("name", sorted(golden.ROWOP_CASES))
def test_checker_matches_reference_golden(name):
    case = golden.ROWOP_CASES[name]
    got = _outputs(OURS[case["op"]], golden.rowop_inputs(case))
    ref = np.load(GOLDEN / f"{name}.npz")
    assert len(got) == len(ref.files)
    for i, g in enumerate(got):
        np.testing.assert_array_equal(g, ref[f"out{i}"], err_msg=f"{name} output {i}")


@pytest.mark.skipif(not (REFERENCE / "references" / "rms_norm.py").exists(), reason="reference checkout absent")
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_checker_matches_reference_live(seed):
    ref = golden.reference_rowop_checkers(REFERENCE)
    cases = [dict(op="rms_norm", m=17, n=4096, dtype="bfloat16", seed=seed),
             dict(op="swiglu_input_quant", m=9, n=1024, seed=seed),
             dict(op="qkv_part_rope", b=1, s=9, heads=4, d=256, q_heads=2, kv_heads=1, nope=128,
                  negative_sin=bool(seed % 2), seed=seed)]
    for case in cases:
        inputs = golden.rowop_inputs(case)
        a = _outputs(OURS[case["op"]], inputs)
        b = _outputs(ref[case["op"]], golden.rowop_inputs(case))
        for i, (x, y) in enumerate(zip(a, b)):
            np.testing.assert_array_equal(x, y, err_msg=f"{case['op']} output {i}")
