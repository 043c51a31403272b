"""ctypes binding of libfa_sm100.so (the C ABI in include/fa_sm100.h).

The library is loaded once, from this package's directory.  There is no
fallback: if the library is missing, every entry point raises RuntimeError.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from .build import lib_path

FA_OK = 0
FA_ERR_ARG = 1
FA_ERR_TMA = 2
FA_ERR_LAUNCH = 3
FA_ERR_DEVICE = 4
FA_ERR_WORKSPACE = 5
FA_ERR_SCRATCH_LIMIT = 6

BWD_DETERMINISTIC = 1

STATUS_TIMEOUT = 1
STATUS_RANGE = 2

DTYPE_F16 = 0
DTYPE_BF16 = 1
_DTYPES = {torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}


def dtype_code(dt: torch.dtype) -> int:
    """FA_DTYPE_* of a torch dtype (fp16 or bf16)."""
    return _DTYPES[dt]

_lock = threading.Lock()
_lib = None

_c_int, _c_float, _vp, _c_size = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


def load() -> ctypes.CDLL:
    """Load libfa_sm100.so (raises RuntimeError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = os.environ.get("FA_SM100_LIB") or lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m flash_attn_volta_b200.build` "
                    "(the CUDA kernels have no fallback)")
            lib = ctypes.CDLL(path)
            lib.fa_sm100_fwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                         _c_float, _c_int, _vp, _vp]
            lib.fa_sm100_fwd.restype = _c_int
            lib.fa_sm100_bwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_size,
                                         _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp,
                                         _vp]
            lib.fa_sm100_bwd.restype = _c_int
            lib.fa_sm100_fwd_ex.argtypes = [_vp] * 5 + [_c_int] * 7 + [_c_float, _c_int, _vp, _vp]
            lib.fa_sm100_fwd_ex.restype = _c_int
            lib.fa_sm100_bwd_ex.argtypes = [_vp] * 10 + [_c_size] + [_c_int] * 7 + [
                _c_float, _c_int, _vp, _vp]
            lib.fa_sm100_bwd_ex.restype = _c_int
            lib.fa_sm100_bwd_flags.argtypes = [_vp] * 10 + [_c_size] + [_c_int] * 7 + [
                _c_float, _c_int, _c_int, _vp, _vp]
            lib.fa_sm100_bwd_flags.restype = _c_int
            lib.fa_sm100_bwd_workspace_bytes_flags.argtypes = [_c_int] * 5
            lib.fa_sm100_bwd_workspace_bytes_flags.restype = _c_size
            lib.fa_sm100_merge.argtypes = [_vp] * 4 + [_c_int] * 6 + [_vp]
            lib.fa_sm100_merge.restype = _c_int
            lib.fa_sm100_bwd_phase.argtypes = [_c_int] + lib.fa_sm100_bwd.argtypes
            lib.fa_sm100_bwd_phase.restype = _c_int
            lib.fa_sm100_bwd_noalloc.argtypes = [_vp] * 9 + [_c_int] * 4 + [_c_float, _c_int,
                                                                             _vp, _vp]
            lib.fa_sm100_bwd_noalloc.restype = _c_int
            lib.fa_sm100_bwd_workspace_bytes.argtypes = [_c_int, _c_int, _c_int, _c_int]
            lib.fa_sm100_bwd_workspace_bytes.restype = _c_size
            lib.fa_sm100_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
            lib.fa_sm100_set_wait_timeout_ns.restype = None
            lib.fa_sm100_set_debug_flags.argtypes = [_c_int]
            lib.fa_sm100_set_debug_flags.restype = None
            lib.fa_sm100_error_string.argtypes = [_c_int]
            lib.fa_sm100_error_string.restype = ctypes.c_char_p
            lib.fa_sm100_abi_version.argtypes = []
            lib.fa_sm100_abi_version.restype = _c_int
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != FA_OK:
        msg = load().fa_sm100_error_string(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (code {rc})")


# ----------------------------------------------------------------- status word
def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 the kernels OR error bits into (bit 0: an on-device wait
    timed out; bit 1: a backward row term was clamped).  One word per device,
    shared with the torch.ops.fav operators."""
    from . import ops
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return ops.status_word(idx)


def status_ptr(idx: int) -> int:
    """Device address of the status word of CUDA device `idx`."""
    return status_word(torch.device("cuda", idx)).data_ptr()


def stream_ptr(idx: int) -> int:
    """cudaStream_t of the current torch stream on CUDA device `idx`."""
    return _raw_stream(idx)


def _raw_stream_fallback(idx: int) -> int:
    return torch.cuda.current_stream(idx).cuda_stream


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None) or _raw_stream_fallback


class on_device:
    """Make CUDA device `idx` current for the block (a no-op when it already is)."""
    __slots__ = ("idx", "prev")

    def __init__(self, idx: int):
        self.idx = idx
        self.prev = -1

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev >= 0:
            torch.cuda.set_device(self.prev)
        return False


def check_status(device: torch.device | None = None) -> None:
    """Synchronise and raise RuntimeError if a kernel on `device` reported an error."""
    from . import ops
    devs = ([device] if device is not None else
            [torch.device("cuda", i) for i in ops.status_devices()])
    for d in devs:
        t = status_word(d)
        v = int(t.item())
        if v:
            t.zero_()
            raise RuntimeError(f"flash_attn_volta_b200 kernel reported status {v} on {d} "
                               "(bit 0: an on-device wait timed out; bit 1: a backward row "
                               "term, LSE/sm_scale or rowsum(O*dO), was beyond the range the "
                               "kernel represents and was clamped)")


_debug_sync = os.environ.get("FA_B200_SYNC_CHECK", "0") == "1"


def debug_sync() -> bool:
    """FA_B200_SYNC_CHECK=1 (read at import): synchronise and check the status
    word after every call."""
    return _debug_sync


_deterministic = os.environ.get("FA_B200_DETERMINISTIC", "0") == "1"


def deterministic_default() -> bool:
    """Default dQ mode of the backward: FA_B200_DETERMINISTIC=1 (read at import)
    selects the separate, bit-reproducible dQ kernel; otherwise dQ partials go
    through L2 reductions."""
    return _deterministic
