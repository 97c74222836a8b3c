"""CPU checks of the C-ABI boundary: the library loads and exports exactly what
include/fuselse_b200.h declares (no compute calls without a GPU)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fuselse_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(?:int|const char\*)\s+(fl_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("fl_lse_f32_fwd", "fl_lse_f32_bwd", "fl_lse_f16_fwd", "fl_intlse_q16_f32",
                 "fl_intlse_q16_i32", "fl_intlse_q10_6_i16", "fl_sparse_f32", "fl_sparse_q16",
                 "fl_lse_combine", "fl_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from fuselse_b200 import _lib
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), f"{name} not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (fl_\w+)", out))
    assert exported == set(declared_functions())


def test_binding_covers_header():
    from fuselse_b200 import _lib
    assert set(_lib.exported_symbols()) == set(declared_functions())


def test_version_and_error_without_gpu():
    from fuselse_b200 import _lib
    L = _lib.lib()
    assert L.fl_version() >= 100
    # argument validation happens before any CUDA call
    st = L.fl_lse_f32_fwd(None, None, -1, 5, 1, None)
    assert st == _lib.FL_ERR_INVALID_ARGUMENT
    assert b"negative" in L.fl_last_error()
    st = L.fl_intlse_q16_f32(ctypes.cast(ctypes.c_void_p(2), ctypes.POINTER(ctypes.c_float)),
                             ctypes.cast(ctypes.c_void_p(16), ctypes.POINTER(ctypes.c_float)),
                             1, 4, 1, None)
    assert st == _lib.FL_ERR_INVALID_ARGUMENT  # misaligned x
    assert _lib.lib().fl_lse_f32_fwd(None, None, 0, 0, 1, None) == _lib.FL_OK  # empty is a no-op


def test_row_counts_checked_before_arithmetic():
    """A row count so large that a byte count formed from it would wrap around
    is rejected before any CUDA call (no GPU needed)."""
    from fuselse_b200 import _lib
    L = _lib.lib()
    fp = ctypes.cast(ctypes.c_void_p(256), ctypes.POINTER(ctypes.c_float))
    for B in ((1 << 60) + 8, (1 << 59), (1 << 62) + 1):
        st = L.fl_lse_vocab_exchange_noalloc(ctypes.c_void_p(256), 0, B, 4, fp, None)
        assert st == _lib.FL_ERR_INVALID_ARGUMENT
        assert b"at most 262112 rows" in L.fl_last_error()
    nbytes = ctypes.c_int64()
    assert L.fl_vocab_exchange_bytes(8, (1 << 60) + 8, ctypes.byref(nbytes)) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_vocab_exchange_bytes(8, 8192, ctypes.byref(nbytes)) == _lib.FL_OK
    assert nbytes.value == 512 + 2 * 8 * 8192 * 8


def test_exchange_wait_limit_setter_without_gpu():
    from fuselse_b200 import _lib
    L = _lib.lib()
    prev = ctypes.c_int64()
    assert L.fl_vocab_exchange_set_wait_limit(100, ctypes.byref(prev)) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_vocab_exchange_set_wait_limit(50_000_000, ctypes.byref(prev)) == _lib.FL_OK
    assert prev.value == 2_000_000_000
    assert L.fl_vocab_exchange_set_wait_limit(prev.value, None) == _lib.FL_OK


@pytest.mark.gpu
def test_library_kernels_are_sm100():
    """The kernels the library loads on the GPU were built for sm_100
    (cudaFuncGetAttributes' binaryVersion; the build targets sm_100a only)."""
    from fuselse_b200 import _lib
    v = ctypes.c_int()
    _lib.call("fl_binary_version", 0, ctypes.byref(v))
    assert v.value == 100, v.value


def test_sparse_bwd_workspace_checks_without_gpu():
    from fuselse_b200 import _lib
    L = _lib.lib()
    nbytes = ctypes.c_int64()
    assert L.fl_sparse_f32_bwd_workspace(1000, 70, 5000, ctypes.byref(nbytes)) == _lib.FL_OK
    # the folded rows, one sign word per 32 columns (each 256-byte aligned),
    # then a partial sum per unit and 64-column group
    r256 = lambda v: (v + 255) // 256 * 256
    assert nbytes.value == r256(1000 * 70 * 4) + r256(1000 * 3 * 4) + 2 * 5000 * 4
    assert L.fl_sparse_f32_bwd_workspace(-1, 70, 0, ctypes.byref(nbytes)) == _lib.FL_ERR_INVALID_ARGUMENT
    # a workspace below that size is refused before any CUDA call
    fp = lambda a: ctypes.cast(ctypes.c_void_p(a), ctypes.POINTER(ctypes.c_float))
    ip = lambda a: ctypes.cast(ctypes.c_void_p(a), ctypes.POINTER(ctypes.c_int64))
    st = L.fl_sparse_f32_bwd(fp(256), fp(512), fp(768), fp(1024), ip(1280), ip(1536), ip(1792),
                             ip(2048), ip(2304), ip(2560), 1, fp(2816), None, 1000, 10, 10, 1, 1,
                             70, 1, ctypes.c_void_p(4096), 1024, None, None)
    assert st == _lib.FL_ERR_INVALID_ARGUMENT
    assert b"workspace" in L.fl_last_error()


def test_ipc_and_query_arguments_checked_without_gpu():
    """The exchange-buffer helpers and the binary-version query reject bad
    arguments before any CUDA call."""
    from fuselse_b200 import _lib
    L = _lib.lib()
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    assert L.fl_ipc_buffer_alloc(-1, 1024, ctypes.byref(ptr), handle) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_alloc(0, 0, ctypes.byref(ptr), handle) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_alloc(0, 1 << 41, ctypes.byref(ptr), handle) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_alloc(0, 1024, None, handle) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_open(0, None, ctypes.byref(ptr)) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_open(-2, handle, ctypes.byref(ptr)) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_close(0, None) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_free(-1, None) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_ipc_buffer_free(0, None) == _lib.FL_OK  # freeing nothing is a no-op
    v = ctypes.c_int()
    assert L.fl_binary_version(-1, ctypes.byref(v)) == _lib.FL_ERR_INVALID_ARGUMENT
    assert L.fl_binary_version(0, None) == _lib.FL_ERR_INVALID_ARGUMENT
