"""The C-ABI library on a host without a GPU: it loads, exports every symbol
include/dq_abi.h declares, and validates arguments before touching CUDA."""
import ctypes as C
import os
import re
import subprocess

import pytest

from dyn_quant import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dq_abi.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DQ_API\s+[\w\s\*]+?\b(dq_\w+)\s*\(", text)))


def test_header_declares_the_exported_list():
    assert declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (dq_\w+)", out))
    assert set(declared_functions()) <= exported
    # nothing else leaks: the kernels' C++ symbols stay hidden
    assert exported == set(declared_functions())


def test_status_strings_and_version():
    assert _lib.status_string(0) == "DQ_OK"
    assert _lib.status_string(_lib.DQ_ERR_CUDA) == "DQ_ERR_CUDA"
    assert _lib.status_string(99) == "DQ_ERR_UNKNOWN"
    L = _lib.lib()
    assert L.dq_version() >= 100
    assert L.dq_max_d_in() >= 28672  # the Llama-2-70B down-projection width


def test_validation_happens_before_any_cuda_call():
    L = _lib.lib()
    ws = (C.c_void_p(256), 1 << 30)  # a well-formed (never dereferenced) workspace argument
    w = _lib.weights(16, 16, 16, 16, None, 16, 100)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, *ws, None) == _lib.DQ_ERR_SHAPE
    w = _lib.weights(16, 16, 16, None, None, 16, 128)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, *ws, None) == _lib.DQ_ERR_INVALID_ARGUMENT
    w = _lib.weights(17, 16, 16, 16, None, 16, 128)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, *ws, None) == _lib.DQ_ERR_ALIGNMENT
    w = _lib.weights(16, 16, 16, 16, None, 16, 1 << 20)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, *ws, None) == _lib.DQ_ERR_UNSUPPORTED
    assert L.dq_split_gemv(None, C.c_void_p(16), C.c_void_p(16), 3.0, *ws, None) == _lib.DQ_ERR_INVALID_ARGUMENT
    w = _lib.weights(16, 16, 16, 16, None, -1, 128)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, *ws, None) == _lib.DQ_ERR_SHAPE
    w = _lib.weights(16, 16, 16, 16, None, 16, 128)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, None, 0, None) == _lib.DQ_ERR_WORKSPACE
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, C.c_void_p(256), 16, None) == _lib.DQ_ERR_WORKSPACE
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, C.c_void_p(272), 1 << 30, None) == _lib.DQ_ERR_ALIGNMENT
    assert L.dq_workspace_bytes(4096, 4096) > 0 and L.dq_workspace_bytes(4096, 100) == 0
    # d_out == 0 is an empty GEMV: nothing to launch
    w = _lib.weights(16, 16, 16, 16, None, 0, 128)
    assert L.dq_split_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, None, 0, None) == _lib.DQ_OK
    assert L.dq_int4_gemv(C.byref(w), C.c_void_p(16), C.c_void_p(16), None, 0, None) == _lib.DQ_OK
    assert L.dq_reference_gemv(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 0, 128, None) == _lib.DQ_OK
    assert L.dq_reference_gemv(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 4, 100, None) == _lib.DQ_ERR_SHAPE
    assert L.dq_quantize(C.c_void_p(16), 4, 100, C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), None) == _lib.DQ_ERR_SHAPE
    assert L.dq_quantize(C.c_void_p(18), 4, 128, C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), None) == _lib.DQ_ERR_ALIGNMENT
    assert L.dq_quantize(None, 4, 128, C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), None) == _lib.DQ_ERR_INVALID_ARGUMENT
    assert L.dq_detect_outliers(None, 128, 3.0, None, None, None, None, None) == _lib.DQ_ERR_INVALID_ARGUMENT
    assert L.dq_detect_outliers(C.c_void_p(16), 100, 3.0, None, None, None, None, None) == _lib.DQ_ERR_SHAPE
    assert L.dq_build_colmajor(C.c_void_p(16), 4, 100, C.c_void_p(16), None) == _lib.DQ_ERR_SHAPE


def test_workspace_sizes_cover_the_column_slabs():
    """Rows of 24576 columns or more may run in column slabs, whose tagged
    partial sums (8 bytes per row and slab after the first) follow the
    workspace's fixed 197376-byte head; a workspace of dq_workspace_bytes
    always has room for them."""
    L = _lib.lib()
    head = 197376
    for d_out in (1024, 4096, 8192):
        n_rb = (d_out + 15) // 16
        assert L.dq_workspace_bytes(d_out, 28672) >= head + n_rb * 3 * 16 * 8  # 4 slabs of 14 chunks
        assert L.dq_workspace_bytes(d_out, 30720) >= head + n_rb * 3 * 16 * 8  # 4 slabs of 15 chunks
    assert L.dq_workspace_bytes(8192, 8192) >= head
    # the grouped batched workspace is one region per problem
    one = L.dq_workspace_bytes_batched_grouped(4096, 14336, 8, 1)
    assert one > 0 and L.dq_workspace_bytes_batched_grouped(4096, 14336, 8, 8) == 8 * one
    assert one % 256 == 0


def test_grouped_validation_happens_before_any_cuda_call():
    L = _lib.lib()
    w = _lib.weights(16, 16, 16, None, 16, 256, 1024, 16)
    ws = 1 << 30
    need = L.dq_workspace_bytes_batched_grouped(256, 1024, 4, 2)
    assert need > 0 and L.dq_workspace_bytes_batched_grouped(256, 1024, 4, 17) == 0
    assert L.dq_workspace_bytes_batched_grouped(256, 100, 4, 2) == 0

    def call(ws_list, xs, ms, wsb=ws, ws_ptr=256):
        return _lib.batched_grouped(ws_list, xs, [16] * len(xs), ms, 3.0, ws_ptr, wsb, None)
    assert call([w, w], [16, 16], [2, 0]) == _lib.DQ_ERR_SHAPE
    assert call([w, w], [16, 16], [2, 17]) == _lib.DQ_ERR_SHAPE
    assert call([], [], []) == _lib.DQ_ERR_SHAPE
    other = _lib.weights(16, 16, 16, None, 16, 256, 2048, 16)
    assert call([w, other], [16, 16], [2, 2]) == _lib.DQ_ERR_SHAPE
    assert call([w, w], [16, 18], [2, 2]) == _lib.DQ_ERR_ALIGNMENT
    assert call([w, w], [16, 16], [2, 4], wsb=need - 256) == _lib.DQ_ERR_WORKSPACE
    no_native = _lib.weights(16, 16, 16, None, 16, 256, 1024, None)
    assert call([w, no_native], [16, 16], [2, 2]) == _lib.DQ_ERR_INVALID_ARGUMENT


def test_check_raises_dqerror():
    with pytest.raises(_lib.DqError) as e:
        _lib.check(_lib.DQ_ERR_SHAPE, "dq_split_gemv")
    assert "DQ_ERR_SHAPE" in str(e.value)
