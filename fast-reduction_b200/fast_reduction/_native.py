"""ctypes binding of libfrx.so (the sm_100a engine; C ABI declared in include/frx.h).

There is no fallback: if the library is missing or fails to load, every entry point raises.
Tensors cross the boundary as raw device pointers plus sizes; the stream is torch's current
stream of the tensors' device, so calls order correctly with surrounding torch work.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# FRX_LIB: a path to the library, or "checked" for the checked build (libfrx_checked.so: buffer
# range checks before every launch, device-side invariant checks).
_NATIVE_DIR = Path(__file__).resolve().parent / "_native"
_LIB_PATH = Path({"": _NATIVE_DIR / "libfrx.so", "checked": _NATIVE_DIR / "libfrx_checked.so"}.get(
    os.environ.get("FRX_LIB", ""), os.environ.get("FRX_LIB", "")))

FRX_OK = 0
FRX_ERR_INVALID_ARG = 1
FRX_ERR_UNSUPPORTED = 2
FRX_ERR_CUDA = 3

FRX_DTYPE_BF16 = 0
FRX_DTYPE_F32 = 1
FRX_DTYPE_F16 = 2

FRX_OUT_ACCUMULATE = 256
FRX_PART_HI = 0
FRX_PART_MID = 1
FRX_PART_LO = 2

FRX_VOCAB_TILE = 256
FRX_PARTIALS_REF_LAYOUT = 1
FRX_IGNORE_NEGATIVE_TARGETS = 2

FRX_STATUS_TIMEOUT_PRODUCER = 1
FRX_STATUS_TIMEOUT_MMA = 2
FRX_STATUS_TIMEOUT_EPILOGUE = 4
FRX_STATUS_BAD_TARGET = 8
FRX_STATUS_DRAIN_TIMEOUT = 16
FRX_STATUS_CHECK_FAILED = 32

_STATUS_NAMES = {
    FRX_STATUS_TIMEOUT_PRODUCER: "TMA producer wait timed out",
    FRX_STATUS_TIMEOUT_MMA: "MMA issuer wait timed out",
    FRX_STATUS_TIMEOUT_EPILOGUE: "epilogue wait timed out",
    FRX_STATUS_BAD_TARGET: "target id outside [0, vocab_size) and not ignore_index",
    FRX_STATUS_DRAIN_TIMEOUT: "in-flight copies did not drain after an abort",
    FRX_STATUS_CHECK_FAILED: "a device-side invariant check of the checked build failed",
}

# Every exported symbol with its ctypes signature: (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F32 = ctypes.c_float
SIGNATURES: dict[str, tuple] = {
    "frx_abi_version": (_I32, []),
    "frx_last_error": (ctypes.c_char_p, []),
    "frx_fwd_partials": (_I32, [_P, _I64, _P, _I64, _I32, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _P,
                                _P]),
    "frx_fwd_partials_tilerel": (_I32, [_P, _I64, _P, _I64, _I32, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P,
                                        _I64, _P, _P]),
    "frx_dlogits_tilerel": (
        _I32,
        [_P, _I64, _P, _I64, _P, _P, _P, _P, _P, _F32, _F32, _P, _I64, _I32, _I64, _I64, _I64, _I64, _P],
    ),
    "frx_finalize": (_I32, [_P, _I64, _I64, _I64, _I32, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P]),
    "frx_dlogits": (
        _I32,
        [_P, _I64, _P, _P, _P, _P, _P, _F32, _F32, _P, _I64, _I32, _I64, _I64, _I64, _I64, _P],
    ),
    "frx_gemm_dhidden": (_I32, [_P, _I64, _P, _I64, _I32, _P, _I64, _I32, _I64, _I64, _I64, _P, _P]),
    "frx_gemm_dweight": (_I32, [_P, _I64, _P, _I64, _I32, _P, _I64, _I32, _I64, _I64, _I64, _P, _P]),
    "frx_gemm_dweight_sms": (_I32, [_P, _I64, _P, _I64, _I32, _P, _I64, _I32, _I64, _I64, _I64, _I32, _P, _P]),
    "frx_fwd_ce_entropy_noalloc": (_I32, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P]),
    "frx_logits_partials": (_I32, [_P, _I32, _I64, _I64, _I64, _P, _I64, _P, _I64, _P]),
    "frx_column_sums": (_I32, [_P, _I32, _I64, _I64, _I64, _P, _P]),
    "frx_gemm_dhidden_multicast": (_I32, [_P, _I64, _P, _I64, _I32, _P, _I64, _I64, _I64, _I64, _P, _P]),
    "frx_split_f32": (_I32, [_P, _I64, _I64, _I64, ctypes.c_uint32, _I32, _P, _I64, _I64, _P]),
    "frx_test_stalled_fwd": (_I32, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _P, _I64, _I32, _I64, _P, _P]),
    "frx_loss_sum": (_I32, [_P, _P, _I64, _F32, _F32, _P, _P]),
    "frx_scale_inplace": (_I32, [_P, _I32, _I64, _P, _P]),
    "frx_check_range": (_I32, [_P, _I64]),
    "frx_clock_probe": (_I32, [_P, _I32, _P]),
}

_lib = None
_lib_lock = threading.Lock()


class FrxError(RuntimeError):
    """A libfrx entry point returned a non-zero status."""


class FrxDeviceError(RuntimeError):
    """A kernel reported a problem through the device status word."""


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Loads libfrx.so once; raises if it is missing (no CPU or library fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise ImportError(
                    f"libfrx.so not found at {_LIB_PATH}; build it with "
                    "`python fast-reduction_b200/build.py` (nvcc, sm_100a)"
                )
            lib = ctypes.CDLL(str(_LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != FRX_OK:
        msg = load().frx_last_error().decode(errors="replace")
        raise FrxError(f"{what} failed (code {rc}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_status_words: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The device int the kernels OR FRX_STATUS_* bits into (one per device, zero-initialised)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def read_status(device: torch.device, reset: bool = True) -> int:
    """Synchronises with the device's status word and returns its bits (optionally clearing)."""
    w = status_word(device)
    val = int(w.item())
    if reset and val:
        w.zero_()
    return val


def raise_on_status(device: torch.device) -> None:
    bits = read_status(device)
    if bits:
        names = [name for bit, name in _STATUS_NAMES.items() if bits & bit]
        raise FrxDeviceError(f"device status 0x{bits:x}: " + "; ".join(names))
