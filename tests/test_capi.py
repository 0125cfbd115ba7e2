"""libtokmix.so: it loads, exports every entry point include/tokmix.h declares, and rejects bad
arguments through its status codes without touching a GPU (CPU-only checks)."""

import ctypes
import pathlib
import re
import subprocess

import pytest

from kernel_opt_agent_b200 import _lib

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "tokmix.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tokmix_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert syms, "no declarations parsed"
    for s in syms:
        assert hasattr(lib, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (tokmix_\w+)", out))
    assert set(syms) <= exported
    assert set(_lib.SIGNATURES) == set(syms)


def test_version():
    assert _lib.version().startswith("tokmix ") and "sm_100a" in _lib.version()


def test_fa2_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # null pointer (non-empty problem)
    rc = lib.tokmix_fa2_fwd(None, p, p, p, 1, 8, 8, 128, 128, 128, 0, 1, 0.1, None, None)
    assert rc == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "null" in _lib.last_error()
    # heads_q not a multiple of heads_kv
    rc = lib.tokmix_fa2_fwd(p, p, p, p, 1, 6, 4, 128, 128, 128, 0, 1, 0.1, None, None)
    assert rc == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "multiple" in _lib.last_error()
    # bad layout / scale / alignment
    assert lib.tokmix_fa2_fwd(p, p, p, p, 1, 8, 8, 128, 128, 128, 7, 1, 0.1, None, None) == 1
    assert lib.tokmix_fa2_fwd(p, p, p, p, 1, 8, 8, 128, 128, 128, 0, 1, -1.0, None, None) == 1
    odd = ctypes.c_void_p(18)
    assert lib.tokmix_fa2_fwd(odd, p, p, p, 1, 8, 8, 128, 128, 128, 0, 1, 0.1, None, None) == 1
    # empty problem is a no-op success
    assert lib.tokmix_fa2_fwd(p, p, p, p, 0, 8, 8, 128, 128, 128, 0, 1, 0.1, None, None) == 0


def test_gdn_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # every call below is rejected (or is a no-op) before anything is launched
    # q k v g beta state out final cu order nseq tokens hk hv dk dv scale io gates status stream
    args = [p, p, p, p, p, None, p, p, p, None, 1, 64, 16, 32, 128, 128, 0.08, 0, None, p, None]
    bad = list(args)
    bad[0] = None
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "null" in _lib.last_error()
    bad = list(args)
    bad[13] = 24  # heads_v not a multiple of heads_k
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[14] = 64  # head dim
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_UNSUPPORTED
    bad = list(args)
    bad[17] = 1  # fp32 io
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_UNSUPPORTED
    bad = list(args)
    bad[19] = None  # status word required
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[3] = bad[4] = None  # g and beta missing without gate inputs
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "null" in _lib.last_error()
    gates = _lib.Stage1Inputs(16, 16, 5, 16, 16)  # unknown dtype
    bad[18] = ctypes.byref(gates)
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "gates" in _lib.last_error()
    gates = _lib.Stage1Inputs(16, None, 0, 16, 16)  # b missing
    bad[18] = ctypes.byref(gates)
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "gates" in _lib.last_error()
    bad = list(args)
    bad[10] = 0  # no sequences: no-op
    assert lib.tokmix_gdn_prefill(*bad) == _lib.TOKMIX_OK


def test_python_wrappers_raise_valueerror_on_cpu_tensors():
    import torch

    from kernel_opt_agent_b200 import flash_attention_2 as fa2
    from kernel_opt_agent_b200 import qwen35moe_gdn_prefill as gdn

    q = torch.zeros(1, 2, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fa2.kernel_fn(q, q, q)
    x = torch.zeros(1, 4, 16, 128)
    y = torch.zeros(1, 4, 32, 128)
    gb = torch.zeros(1, 4, 32)
    with pytest.raises(ValueError):
        gdn.kernel_fn(x, x, y, gb, gb, torch.zeros(1, 32, 128, 128))


def test_gdn_split_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    need = lib.tokmix_gdn_split_workspace_bytes(32, 32)
    assert need >= 32 * 32 * 4 * 1024 and need % 16 == 0  # records plus one flag word per record
    assert lib.tokmix_gdn_split_workspace_bytes(-1, 32) == -1
    # q k v g beta state out final checkpoints cu chunk_base order nseq tokens chunks hk hv dk dv scale io gates ws
    # ws_bytes status stream
    args = [p, p, p, p, p, None, p, p, None, p, p, None, 1, 2048, 32, 16, 32, 128, 128, 0.08, 0, None, p, need, p, None]
    bad = list(args)
    bad[10] = None  # chunk_base
    assert lib.tokmix_gdn_prefill_split(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "null" in _lib.last_error()
    bad = list(args)
    bad[23] = need - 16  # workspace too small
    assert lib.tokmix_gdn_prefill_split(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "workspace" in _lib.last_error()
    bad = list(args)
    bad[17] = 64  # head dim
    assert lib.tokmix_gdn_prefill_split(*bad) == _lib.TOKMIX_ERR_UNSUPPORTED
    bad = list(args)
    bad[20] = 1  # fp32 io
    assert lib.tokmix_gdn_prefill_split(*bad) == _lib.TOKMIX_ERR_UNSUPPORTED
    bad = list(args)
    bad[12] = 0  # no sequences: no-op
    assert lib.tokmix_gdn_prefill_split(*bad) == _lib.TOKMIX_OK


def test_gdn_decode_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # q k v g beta state_in state_out out batch hk hv dk dv scale io stream
    args = [p, p, p, p, p, None, p, p, 4, 16, 32, 128, 128, 0.08, 0, None]
    bad = list(args)
    bad[6] = None  # state_out
    assert lib.tokmix_gdn_decode(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "null" in _lib.last_error()
    bad = list(args)
    bad[10] = 24  # heads_v not a multiple of heads_k
    assert lib.tokmix_gdn_decode(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[11] = 64  # head dim
    assert lib.tokmix_gdn_decode(*bad) == _lib.TOKMIX_ERR_UNSUPPORTED
    bad = list(args)
    bad[14] = 1  # fp32 io
    assert lib.tokmix_gdn_decode(*bad) == _lib.TOKMIX_ERR_UNSUPPORTED
    bad = list(args)
    bad[1] = ctypes.c_void_p(24)  # misaligned k
    assert lib.tokmix_gdn_decode(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "aligned" in _lib.last_error()
    bad = list(args)
    bad[8] = 0  # empty batch: no-op
    assert lib.tokmix_gdn_decode(*bad) == _lib.TOKMIX_OK


def test_l2norm_rows_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.tokmix_l2norm_rows(p, 0, p, 10, 64, 1e-6, None) == _lib.TOKMIX_ERR_UNSUPPORTED  # row length
    assert lib.tokmix_l2norm_rows(p, 7, p, 10, 128, 1e-6, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT  # dtype
    assert lib.tokmix_l2norm_rows(p, 0, None, 10, 128, 1e-6, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_l2norm_rows(p, 0, p, -1, 128, 1e-6, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_l2norm_rows(p, 0, p, 10, 128, -1.0, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_l2norm_rows(p, 0, p, 0, 128, 1e-6, None) == _lib.TOKMIX_OK  # nothing to do


def test_gdn_gates_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.tokmix_gdn_gates(p, p, 1, p, p, p, p, 10, 0, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT  # heads
    assert lib.tokmix_gdn_gates(p, p, 5, p, p, p, p, 10, 32, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT  # dtype
    assert lib.tokmix_gdn_gates(p, p, 1, None, p, p, p, 10, 32, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_gdn_gates(p, p, 1, p, p, p, p, 0, 32, None) == _lib.TOKMIX_OK  # nothing to do



def test_rms_norm_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    bf16, fp16 = _lib.DTYPE_BF16, _lib.DTYPE_FP16
    assert lib.tokmix_rms_norm(p, p, p, 10, 100, bf16, 1e-6, None) == _lib.TOKMIX_ERR_UNSUPPORTED  # n % 8
    assert lib.tokmix_rms_norm(p, p, p, 10, 128, 1, 1e-6, None) == _lib.TOKMIX_ERR_UNSUPPORTED  # fp32
    assert lib.tokmix_rms_norm(p, p, p, -1, 128, bf16, 1e-6, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_rms_norm(p, p, p, 10, 128, fp16, -1.0, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_rms_norm(p, None, p, 10, 128, bf16, 1e-6, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_rms_norm(p, p, ctypes.c_void_p(24), 10, 128, bf16, 1e-6, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_rms_norm(p, p, p, 0, 128, bf16, 1e-6, None) == _lib.TOKMIX_OK  # nothing to do


def test_swiglu_input_quant_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.tokmix_swiglu_input_quant(p, p, p, p, 4, 96, 1e-15, None) == _lib.TOKMIX_ERR_UNSUPPORTED  # n % 128
    assert lib.tokmix_swiglu_input_quant(p, p, p, p, -1, 128, 1e-15, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_swiglu_input_quant(p, p, p, p, 4, 128, 0.0, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT  # eps
    assert lib.tokmix_swiglu_input_quant(p, p, None, p, 4, 128, 1e-15, None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert lib.tokmix_swiglu_input_quant(p, p, p, p, 0, 128, 1e-15, None) == _lib.TOKMIX_OK


def test_qkv_part_rope_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    ok = [p, p, p, p, 1, 16, 12, 256, 10, 1, 192, 0, None]

    def call(**changes):
        args = list(ok)
        names = ["qkv", "cos", "sin", "out", "batch", "seq", "heads", "head_dim", "q_heads", "kv_heads", "nope_dim",
                 "negative_sin", "stream"]
        for key, val in changes.items():
            args[names.index(key)] = val
        return lib.tokmix_qkv_part_rope(*args)

    assert call(q_heads=12) == _lib.TOKMIX_ERR_INVALID_ARGUMENT  # q_heads + kv_heads > heads
    assert call(nope_dim=196) == _lib.TOKMIX_ERR_UNSUPPORTED
    assert call(nope_dim=264) == _lib.TOKMIX_ERR_UNSUPPORTED  # nope_dim > head_dim
    assert call(batch=-1) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert call(sin=None) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert call(out=ctypes.c_void_p(24)) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    assert call(seq=0) == _lib.TOKMIX_OK


def test_gdn_segmented_rejects_bad_arguments():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    cu = (ctypes.c_int32 * 3)(0, 5000, 9000)
    need = lib.tokmix_gdn_segmented_workspace_bytes(cu, 2, 32, 16)
    assert need > 0 and need % 256 == 0
    assert lib.tokmix_gdn_segmented_plan_bytes(cu, 2, 32, 16) > 0
    assert lib.tokmix_gdn_segmented_workspace_bytes(cu, 2, 32, 0) == -1
    backwards = (ctypes.c_int32 * 3)(0, 5000, 4000)
    assert lib.tokmix_gdn_segmented_workspace_bytes(backwards, 2, 32, 16) == -1
    chunks = (5000 + 63) // 64 + (4000 + 63) // 64
    # q k v g beta state out final cu chunk_base cu_host nseq tokens chunks hk hv dk dv scale io gates seg plan ws
    # ws_bytes status stream
    args = [p, p, p, p, p, None, p, p, p, p, cu, 2, 9000, chunks, 16, 32, 128, 128, 0.08, 0, None, 16, None, p, need,
            p, None]
    bad = list(args)
    bad[13] = chunks + 1  # chunk count disagrees with the host offsets
    assert lib.tokmix_gdn_prefill_segmented(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[24] = need - 256  # workspace too small
    assert lib.tokmix_gdn_prefill_segmented(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT and "workspace" in _lib.last_error()
    bad = list(args)
    bad[21] = 0  # segment length
    assert lib.tokmix_gdn_prefill_segmented(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[10] = backwards
    assert lib.tokmix_gdn_prefill_segmented(*bad) == _lib.TOKMIX_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[11] = 0  # no sequences: no-op
    assert lib.tokmix_gdn_prefill_segmented(*bad) == _lib.TOKMIX_OK
