"""ctypes binding of libmea.so (declared in include/mea.h).

The library is built in-tree (``python -m memory_efficient_attn_layer_b200.build``)
and loaded from next to this file.  There is no fallback: if the library is
missing or the GPU is not an sm_100 part, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmea.so")
HEADER_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mea.h")

MEA_OK = 0
ERROR_NAMES = {
    1: "MEA_ERR_INVALID_ARGUMENT", 2: "MEA_ERR_UNSUPPORTED_SHAPE", 3: "MEA_ERR_ALIGNMENT",
    4: "MEA_ERR_CUDA", 5: "MEA_ERR_DEVICE_TIMEOUT", 6: "MEA_ERR_UNSUPPORTED_DEVICE", 7: "MEA_ERR_WORKSPACE",
}


class MeaBlockDims(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int), ("T", ctypes.c_int), ("C", ctypes.c_int), ("H", ctypes.c_int),
                ("N", ctypes.c_int), ("T_max", ctypes.c_int), ("eps", ctypes.c_float)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_F = ctypes.c_float
_DB = ctypes.c_double
_S = ctypes.c_size_t
_D = ctypes.POINTER(MeaBlockDims)

# name -> (restype, argtypes); mirrors include/mea.h
SIGNATURES = {
    "mea_version": (_I, []),
    "mea_last_error_string": (ctypes.c_char_p, []),
    "mea_device_check": (_I, []),
    "mea_read_status": (_I, [_P, ctypes.POINTER(_I), _P]),
    "mea_forward_workspace_size": (_S, [_D]),
    "mea_block_forward": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P, _P]),
    "mea_backward_workspace_size": (_S, [_D]),
    "mea_block_backward": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                _P, _S, _P, _P]),
    "mea_block_backward_ex": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _S, _P, _P, _P, _P]),
    "mea_block_forward_save_o": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P, _P]),
    "mea_block_backward_from_o": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       _P, _P, _P, _P, _S, _P, _P, _P, _P]),
    "mea_rmsnorm_forward": (_I, [_I, _I, _F, _P, _P, _P, _P]),
    "mea_qkvg_forward": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "mea_attention_forward": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "mea_gemm": (_I, [_I, _I, _I, _P, _LL, _I, _P, _LL, _I, _P, _LL, _I, _P, _P]),
    "mea_gemm_e4m3": (_I, [_I, _I, _I, _P, _LL, _P, _LL, _P, _LL, _I, _P, _P]),
    "mea_gate_backward": (_I, [_D, _P, _P, _P, _P, _P, _P, _LL, _P, _P, _P]),
    "mea_attention_backward": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _LL, _P, _P]),
    "mea_qk_norm_rope_backward": (_I, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _LL, _P, _P, _P]),
    "mea_rmsnorm_backward": (_I, [_I, _I, _P, _P, _P, _P, _P]),
    "mea_attention_backward_noalloc": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _LL, _P, _P]),
    "mea_adamw_step": (_I, [_LL, _P, _P, _P, _P, _P, _DB, _DB, _DB, _DB, _DB, _F, _I, _P]),
    "mea_selftest_wait": (_I, [_P, ctypes.c_ulonglong, _I, _P]),
    "mea_profile_enable": (_I, [_I]),
    "mea_profile_read": (_I, [_I, ctypes.POINTER(_F), ctypes.POINTER(_I)]),
    "mea_profile_stage_name": (ctypes.c_char_p, [_I]),
}

_lib = None
_lock = threading.Lock()


def header_symbols() -> list:
    """Names of the functions declared in include/mea.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mea_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load libmea.so once and declare its signatures."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libmea.so not found at {LIB_PATH}; build it with "
                        "`python -m memory_efficient_attn_layer_b200.build`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


class MeaError(RuntimeError):
    """A non-zero status from libmea; ``code`` is the MEA_ERR_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != MEA_OK:
        raise MeaError(rc, lib().mea_last_error_string().decode(errors="replace"))


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


MEA_ERR_DEVICE_TIMEOUT = 5
_checked_devices = set()


class _StatusWatch:
    """Per-device failure reporting without a per-call synchronisation.

    ``word`` is the device int32 the kernels write when a bounded wait gives
    up (0 = ok).  After every library call the word is copied asynchronously
    into pinned host memory on the calling stream and an event is recorded
    behind the copy; the next call (or check_device_status) looks at the copy
    once that event has completed, so a timeout surfaces as a MeaError at the
    first call after the failing one whose copy has landed, without ever
    blocking the host on the GPU."""

    def __init__(self, device: torch.device):
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None

    def note(self) -> None:
        self.host.copy_(self.word, non_blocking=True)
        if self.event is None:
            self.event = torch.cuda.Event()
        self.event.record()

    def take(self, block: bool) -> int:
        """The last copied value (0 when none has landed yet); clears a reported timeout."""
        if self.event is None:
            return 0
        if block:
            self.event.synchronize()
        elif not self.event.query():
            return 0
        v = int(self.host[0])
        if v != 0:
            self.word.zero_()
            self.host[0] = 0
            self.event = None
        return v


_watch = {}


def _device_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _watcher(device: torch.device) -> _StatusWatch:
    idx = _device_index(device)
    w = _watch.get(idx)
    if w is None:
        with torch.cuda.device(idx):
            w = _StatusWatch(torch.device("cuda", idx))
        _watch[idx] = w
    return w


def status_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels write when a bounded wait gives up."""
    return _watcher(device).word


def _timeout_error(v: int, when: str) -> MeaError:
    return MeaError(MEA_ERR_DEVICE_TIMEOUT, f"device wait timed out (kernel {(v >> 8) & 0xFF}, site "
                                            f"{(v >> 16) & 0xFFFF}) {when}")


def note_status(device: torch.device) -> None:
    """Queue the asynchronous host copy of the status word behind the work just
    launched on the current stream (no synchronisation)."""
    _watcher(device).note()


def poll_status(device: torch.device) -> None:
    """Raise MeaError(MEA_ERR_DEVICE_TIMEOUT) if the last status copy that has
    already landed reports a timeout; never blocks."""
    v = _watcher(device).take(block=False)
    if v != 0:
        raise _timeout_error(v, "in an earlier call")


def check_device_status(device: torch.device | None = None) -> None:
    """Wait for the last status copy of `device` (default: the current one) and
    raise MeaError(MEA_ERR_DEVICE_TIMEOUT) if any kernel launched before it gave
    up a bounded wait.  Call it where the caller synchronises anyway (end of an
    epoch, before a checkpoint) to see a timeout of the very last call."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    v = _watcher(dev).take(block=True)
    if v != 0:
        raise _timeout_error(v, "in an earlier call")


def read_status(device: torch.device) -> int:
    """Synchronises the current stream and raises MeaError if a kernel timed out."""
    w = _watcher(device)
    out = ctypes.c_int(0)
    rc = lib().mea_read_status(ctypes.c_void_p(w.word.data_ptr()), ctypes.byref(out),
                               ctypes.c_void_p(stream_ptr(device)))
    if rc != MEA_OK:
        w.word.zero_()
        w.host[0] = 0
        w.event = None
        check(rc)
    return out.value


def require_device(device: torch.device) -> None:
    """Raises unless `device` is a CUDA sm_100 device (checked once per device)."""
    if device.type != "cuda":
        raise RuntimeError("memory_efficient_attn_layer_b200 runs on CUDA (sm_100a) tensors only; "
                           f"got a tensor on {device}")
    idx = _device_index(device)
    if idx in _checked_devices:
        return
    with torch.cuda.device(idx):
        check(lib().mea_device_check())
    _checked_devices.add(idx)


def profile_enable(on: bool = True) -> None:
    """Start (or stop) per-stage CUDA-event timing inside the block calls."""
    check(lib().mea_profile_enable(1 if on else 0))


def profile_read() -> dict:
    """{stage name: (total ms, launches)} since the last enable/read; syncs."""
    n = 32
    ms = (_F * n)()
    cnt = (_I * n)()
    k = lib().mea_profile_read(n, ms, cnt)
    if k < 0:
        check(k)
    return {lib().mea_profile_stage_name(i).decode(): (ms[i], cnt[i]) for i in range(k) if cnt[i]}
