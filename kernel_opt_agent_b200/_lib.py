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
import os
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
                                _VP, _VP]),
    "tokmix_gdn_prefill_noalloc": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _F, _I, _VP,
                                        _VP]),
    "tokmix_gdn_prefill_split": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I,
                                      _I, _I, _F, _I, _VP, _VP, ctypes.c_longlong, _VP, _VP]),
    "tokmix_gdn_noalloc_status": (_I, [_VP, _I]),
    "tokmix_gdn_prefill_segmented": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I,
                                          _I, _I, _F, _I, _VP, _I, _VP, _VP, ctypes.c_longlong, _VP, _VP]),
    "tokmix_gdn_segmented_workspace_bytes": (ctypes.c_longlong, [_VP, _I, _I, _I]),
    "tokmix_gdn_segmented_plan_bytes": (ctypes.c_longlong, [_VP, _I, _I, _I]),
    "tokmix_gdn_segmented_plan": (_I, [_VP, _I, _I, _I, _VP, ctypes.c_longlong]),
    "tokmix_gdn_split_workspace_bytes": (ctypes.c_longlong, [_I, _I]),
    "tokmix_gdn_decode": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _F, _I, _VP]),
    "tokmix_l2norm_rows": (_I, [_VP, _I, _VP, ctypes.c_longlong, _I, _F, _VP]),
    "tokmix_gdn_gates": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, ctypes.c_longlong, _I, _VP]),
    "tokmix_rms_norm": (_I, [_VP, _VP, _VP, _I, _I, _I, _F, _VP]),
    "tokmix_swiglu_input_quant": (_I, [_VP, _VP, _VP, _VP, _I, _I, _F, _VP]),
    "tokmix_qkv_part_rope": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _I, _I, _VP]),
    "tokmix_selftest_wait_timeout": (_I, [_I, ctypes.c_longlong, _VP, _VP, _VP, _VP]),
    "tokmix_last_error": (ctypes.c_char_p, []),
    "tokmix_version": (ctypes.c_char_p, []),
}

class Stage1Inputs(ctypes.Structure):
    """tokmix_gdn_stage1: the gate projections and q/k normalisation the GDN kernels do in stage 1."""

    _fields_ = [("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("dtype", ctypes.c_int),
                ("a_log", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p), ("qk_l2norm", ctypes.c_int),
                ("l2norm_eps", ctypes.c_float), ("k_normed", ctypes.c_void_p)]


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


def _raise_for(val: int, what: str) -> None:
    reasons = ", ".join(txt for bit, txt in DEV_STATUS_BITS.items() if val & bit) or f"0x{val:x}"
    raise TokmixDeviceError(f"{what}: device status 0x{val:x} ({reasons})")


def raise_on_device_status(word: torch.Tensor, what: str) -> None:
    """Reads the status word (this synchronises the stream) and raises TokmixDeviceError if a
    kernel set a bit; the word is cleared first."""
    val = int(word.item()) & 0xFFFFFFFF
    if val:
        word.zero_()
        _raise_for(val, what)


# How the plugin modules check the device status word after each launch:
#   "async" (default) -- without a synchronisation: a copy of the word to pinned host memory is
#                        queued on a side stream behind the launch, and the next call (or
#                        check_device_status) raises TokmixDeviceError once that copy shows a bit;
#   "sync"            -- synchronise and check after every call;
#   "off"             -- only explicit check_device_status calls look at the word.
# TOKMIX_CHECK_STATUS=1 selects "sync", =0 "off".
_STATUS_MODE = {"1": "sync", "0": "off"}.get(os.environ.get("TOKMIX_CHECK_STATUS", ""), "async")


class _StatusMonitor:
    """Non-blocking watch of one device's status word (see _STATUS_MODE)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.side = torch.cuda.Stream(device)
        self.copied = None  # event recorded after the copy in flight, if any
        self.what = ""

    def poll(self) -> None:
        """Raises if the last completed copy shows a bit (and clears the word)."""
        if self.copied is not None and self.copied.query():
            self.copied = None
            val = int(self.host[0]) & 0xFFFFFFFF
            if val:
                self.host.zero_()
                status_word(self.device).zero_()
                _raise_for(val, self.what)

    def after_launch(self, what: str) -> None:
        self.poll()
        if self.copied is not None:
            return  # one copy in flight at a time; it covers every launch before it
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.side.wait_event(ev)
        with torch.cuda.stream(self.side):
            self.host.copy_(status_word(self.device), non_blocking=True)
        self.copied = torch.cuda.Event()
        self.copied.record(self.side)
        self.what = what


_monitors: dict[int, _StatusMonitor] = {}


def after_launch(device: torch.device, what: str) -> None:
    """Status check after a launch that was given status_word(device), per _STATUS_MODE."""
    if _STATUS_MODE == "off":
        return
    if _STATUS_MODE == "sync":
        raise_on_device_status(status_word(device), what)
        return
    if torch.cuda.is_current_stream_capturing():
        return  # no side-stream work inside a graph capture; check_device_status still works
    idx = device.index if device.index is not None else torch.cuda.current_device()
    m = _monitors.get(idx)
    if m is None:
        m = _monitors[idx] = _StatusMonitor(torch.device("cuda", idx))
    m.after_launch(what)


def check_status(device: torch.device, what: str) -> None:
    """Synchronise and raise if any kernel given status_word(device) reported a device-side
    timeout (also drops a pending asynchronous check, which this one covers)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    m = _monitors.get(idx)
    if m is not None:
        m.copied = None
    raise_on_device_status(status_word(torch.device("cuda", idx)), what)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
