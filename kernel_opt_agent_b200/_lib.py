"""ctypes binding of libtokmix.so (declared in include/tokmix.h).

The library is the only compute path: there is no CPU or PyTorch fallback.  If the shared
object is missing or the device is not a B200 the calls raise.  Errors map the way the
reference's plugin modules report them: bad shapes / dtypes / devices raise ``ValueError``
(``kernels_optimized/flash_attention_2.py:110-125``), launch or device failures raise
``RuntimeError`` (the reference's ``TORCH_CHECK`` after launch,
``kernels_optimized/flash_attention_2.cu:1255-1256``).
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libtokmix.so"

TOKMIX_OK = 0
TOKMIX_ERR_INVALID_ARGUMENT = 1
TOKMIX_ERR_UNSUPPORTED = 2
TOKMIX_ERR_LAUNCH = 3
TOKMIX_ERR_DEVICE = 4

LAYOUT_BHSD = 0
LAYOUT_BSHD = 1
DTYPE_BF16 = 0
DTYPE_FP32 = 1
DTYPE_FP16 = 2

DEV_STATUS_BITS = {
    0x1: "a TMA load never completed",
    0x2: "a tensor-core MMA commit never arrived",
    0x4: "a pipeline hand-off between warps never arrived",
    0x8: "a kernel-side argument check failed",
}

# every exported symbol of include/tokmix.h with its ctypes signature
_VP = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "tokmix_fa2_fwd": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _I, _I, _F, _VP, _VP]),
    "tokmix_gdn_prefill": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _F, _I, _VP,
                                _VP]),
    "tokmix_gdn_prefill_noalloc": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _F, _I, _VP,
                                        _VP]),
    "tokmix_gdn_prefill_split": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I,
                                      _I, _I, _F, _I, _VP, ctypes.c_longlong, _VP, _VP]),
    "tokmix_gdn_split_workspace_bytes": (ctypes.c_longlong, [_I, _I]),
    "tokmix_gdn_decode": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _F, _I, _VP]),
    "tokmix_l2norm_rows": (_I, [_VP, _I, _VP, ctypes.c_longlong, _I, _F, _VP]),
    "tokmix_gdn_gates": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, ctypes.c_longlong, _I, _VP]),
    "tokmix_rms_norm": (_I, [_VP, _VP, _VP, _I, _I, _I, _F, _VP]),
    "tokmix_swiglu_input_quant": (_I, [_VP, _VP, _VP, _VP, _I, _I, _F, _VP]),
    "tokmix_qkv_part_rope": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _I, _I, _VP]),
    "tokmix_last_error": (ctypes.c_char_p, []),
    "tokmix_version": (ctypes.c_char_p, []),
}

_lib = None
_lock = threading.Lock()
_status_words: dict[int, torch.Tensor] = {}


class TokmixDeviceError(RuntimeError):
    """A kernel reported a device-side status bit (a bounded wait ran out)."""


def load() -> ctypes.CDLL:
    """Load libtokmix.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise FileNotFoundError(
                        f"{LIB_PATH} is missing; build it with `python -m kernel_opt_agent_b200.build`")
                lib = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def last_error() -> str:
    return load().tokmix_last_error().decode()


def version() -> str:
    return load().tokmix_version().decode()


def check(rc: int, what: str) -> None:
    if rc == TOKMIX_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == TOKMIX_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def status_word(device: torch.device) -> torch.Tensor:
    """A zeroed device uint32 status word for `device` (one per device, reused)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def raise_on_device_status(word: torch.Tensor, what: str) -> None:
    """Synchronise-free check helper: reads the status word (this synchronises the stream)."""
    val = int(word.item()) & 0xFFFFFFFF
    if val:
        word.zero_()
        reasons = ", ".join(txt for bit, txt in DEV_STATUS_BITS.items() if val & bit) or f"0x{val:x}"
        raise TokmixDeviceError(f"{what}: device status 0x{val:x} ({reasons})")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
