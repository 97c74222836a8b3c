"""ctypes binding of libfuselse_b200.so (the C ABI declared in include/fuselse_b200.h).

The library is loaded from the package directory, never from a system path.
If it is missing, every call raises: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int16, c_int32, c_int64, c_uint16, c_void_p
from pathlib import Path

LIB_PATH = Path(os.environ.get("FUSELSE_B200_LIB", Path(__file__).resolve().parent / "libfuselse_b200.so"))

FL_OK = 0
FL_ERR_INVALID_ARGUMENT = 1
FL_ERR_CUDA = 2
FL_ERR_UNSUPPORTED = 3

_fp = POINTER(c_float)
_stream = c_void_p

# name -> argument types (all return int status)
SIGNATURES = {
    "fl_lse_f32_fwd": [_fp, _fp, c_int64, c_int64, c_int, _stream],
    "fl_lse_f32_bwd": [_fp, _fp, _fp, _fp, c_int64, c_int64, _stream],
    "fl_lse_f32_fwd_strided": [_fp, _fp, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, _stream],
    "fl_lse_f32_bwd_strided": [_fp, _fp, _fp, _fp, c_int64, c_int64, c_int64, c_int64, c_int64,
                               _stream],
    "fl_lse_f32_fwd_dim": [_fp, _fp, c_int64, c_int64, c_int64, c_int, _stream],
    "fl_lse_f32_bwd_dim": [_fp, _fp, _fp, _fp, c_int64, c_int64, c_int64, _stream],
    "fl_lse_f16_fwd": [POINTER(c_uint16), _fp, c_int64, c_int64, _stream],
    "fl_selective_logsoftmax_f32": [_fp, POINTER(c_int64), _fp, _fp, c_int64, c_int64, c_int,
                                    POINTER(c_int), _stream],
    "fl_selective_logsoftmax_f16": [POINTER(c_uint16), POINTER(c_int64), _fp, _fp, c_int64, c_int64,
                                    POINTER(c_int), _stream],
    "fl_selective_logsoftmax_bwd": [_fp, _fp, _fp, POINTER(c_int64), _fp, c_int64, c_int64, _stream],
    "fl_selective_logsoftmax_f32_strided": [_fp, POINTER(c_int64), _fp, _fp, c_int64, c_int64, c_int64,
                                            c_int64, c_int64, c_int, POINTER(c_int), _stream],
    "fl_selective_logsoftmax_bwd_strided": [_fp, _fp, _fp, POINTER(c_int64), _fp, c_int64, c_int64,
                                            c_int64, c_int64, c_int64, _stream],
    "fl_lse_f32_partial": [_fp, _fp, c_int64, c_int64, _stream],
    "fl_lse_f16_partial": [POINTER(c_uint16), _fp, c_int64, c_int64, _stream],
    "fl_lse_combine": [_fp, _fp, c_int64, c_int64, _stream],
    "fl_intlse_q16_f32": [_fp, _fp, c_int64, c_int64, c_int, _stream],
    "fl_intlse_q16_i32": [POINTER(c_int32), _fp, c_int64, c_int64, c_int, _stream],
    "fl_intlse_q10_6_i16": [POINTER(c_int16), _fp, c_int64, c_int64, _stream],
    "fl_sparse_f32": [_fp, _fp, _fp, POINTER(c_int64), POINTER(c_int64), POINTER(c_int64),
                      c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                      POINTER(c_int), _stream],
    "fl_sparse_q16": [_fp, _fp, _fp, POINTER(c_int64), POINTER(c_int64), POINTER(c_int64),
                      c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                      POINTER(c_int), _stream],
    "fl_sparse_log_weights": [_fp, _fp, c_int64, _stream],
    "fl_sparse_f32_bwd": [_fp, _fp, _fp, _fp, POINTER(c_int64), POINTER(c_int64), POINTER(c_int64),
                          POINTER(c_int64), POINTER(c_int64), POINTER(c_int64), c_int64, _fp, _fp,
                          c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                          c_void_p, c_int64, POINTER(c_int), _stream],
    "fl_sparse_f32_bwd_workspace": [c_int64, c_int64, c_int64, POINTER(c_int64)],
    "fl_vocab_exchange_bytes": [c_int64, c_int64, POINTER(c_int64)],
    "fl_lse_vocab_exchange": [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int,
                              _fp, _stream],
    "fl_lse_vocab_exchange_noalloc": [c_void_p, c_int, c_int64, c_int64, _fp, _stream],
    "fl_vocab_exchange_set_wait_limit": [c_int64, POINTER(c_int64)],
    "fl_ipc_buffer_alloc": [c_int, c_int64, POINTER(c_void_p), c_void_p],
    "fl_ipc_buffer_open": [c_int, c_void_p, POINTER(c_void_p)],
    "fl_ipc_buffer_close": [c_int, c_void_p],
    "fl_ipc_buffer_free": [c_int, c_void_p],
    "fl_binary_version": [c_int, POINTER(c_int)],
}


class FuseLSEError(RuntimeError):
    """A non-zero status from the C ABI (subclass of RuntimeError, like TORCH_CHECK)."""

    def __init__(self, func: str, status: int, message: str):
        super().__init__(f"{func}: {message or 'error'} (status {status})")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"fuselse_b200: native library {LIB_PATH} is missing; build it with "
                "`python -m fuselse_b200.build` (there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = argtypes
            f.restype = c_int
        L.fl_last_error.argtypes = []
        L.fl_last_error.restype = c_char_p
        L.fl_version.argtypes = []
        L.fl_version.restype = c_int
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    st = getattr(lib(), name)(*args)
    if st != FL_OK:
        msg = lib().fl_last_error().decode(errors="replace")
        raise FuseLSEError(name, st, msg)


def ptr(t, ctype=c_float):
    """Typed pointer to a tensor's data (None for an empty tensor)."""
    if t is None or t.numel() == 0:
        return None
    return ctypes.cast(t.data_ptr(), POINTER(ctype))


def exported_symbols() -> list[str]:
    return ["fl_last_error", "fl_version", *SIGNATURES]
