"""ctypes binding of the C ABI in include/dq_abi.h (libdq_b200.so).

This is the language-neutral boundary: plain pointers, sizes, a status code.
It is what a non-Python caller binds (cgo, JNI, N-API, ...); the Python API in
dyn_quant/__init__.py goes through the torch extension dyn_quant._C, which
calls the same library.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdq_b200.so")

DQ_OK = 0
DQ_ERR_INVALID_ARGUMENT = 1
DQ_ERR_SHAPE = 2
DQ_ERR_ALIGNMENT = 3
DQ_ERR_UNSUPPORTED = 4
DQ_ERR_CUDA = 5
DQ_ERR_WORKSPACE = 6

# Every symbol include/dq_abi.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "dq_status_string",
    "dq_last_cuda_error",
    "dq_version",
    "dq_max_d_in",
    "dq_quantize",
    "dq_build_colmajor",
    "dq_split_gemv",
    "dq_split_gemv_noalloc",
    "dq_reset_noalloc_workspace",
    "dq_split_gemv_batched",
    "dq_workspace_bytes_batched",
    "dq_split_gemv_batched_grouped",
    "dq_workspace_bytes_batched_grouped",
    "dq_silu_mul",
    "dq_silu_mul_pairs",
    "dq_moe_combine",
    "dq_int4_gemv",
    "dq_reference_gemv",
    "dq_detect_outliers",
    "dq_native_bytes",
    "dq_build_native",
    "dq_read_device_error",
    "dq_workspace_bytes",
    "dq_reset_workspace",
    "dq_gather_region_bytes",
    "dq_split_gemv_gather",
    "dq_device_alloc",
    "dq_device_free",
    "dq_ipc_handle",
    "dq_ipc_open",
    "dq_ipc_close",
)

MAX_GATHER_RANKS = 8  # DQ_MAX_GATHER_RANKS
MAX_BATCH = 16        # vectors of one batched split GEMV call
MAX_GROUPS = 16       # problems of one grouped batched call


class DqWeights(C.Structure):
    """dq_weights_t (include/dq_abi.h)."""

    _fields_ = [
        ("packed", C.c_void_p),
        ("scales", C.c_void_p),
        ("zeros", C.c_void_p),
        ("fp16", C.c_void_p),
        ("fp16_cm", C.c_void_p),
        ("native", C.c_void_p),
        ("d_out", C.c_int32),
        ("d_in", C.c_int32),
    ]


class DqGather(C.Structure):
    """dq_gather_t (include/dq_abi.h)."""

    _fields_ = [
        ("rank", C.c_int32),
        ("world", C.c_int32),
        ("rows_per", C.c_int32),
        ("d_total", C.c_int32),
        ("region", C.c_void_p * MAX_GATHER_RANKS),
    ]


class DqError(RuntimeError):
    def __init__(self, status: int, what: str, cuda_error: int = 0):
        self.status = status
        self.cuda_error = cuda_error
        msg = f"{what} failed: {status_string(status)}"
        if status == DQ_ERR_CUDA:
            msg += f" (cudaError {cuda_error})"
        super().__init__(msg)


_lib = None


def lib() -> C.CDLL:
    """Load libdq_b200.so; raises if it has not been built (there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} not found: build it with `python dyn-quant_b200/build.py` "
                "(the dyn-quant kernels have no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        P, i32, f32, st = C.c_void_p, C.c_int32, C.c_float, C.c_int
        L.dq_status_string.restype = C.c_char_p
        L.dq_status_string.argtypes = [st]
        L.dq_last_cuda_error.restype = C.c_int
        L.dq_version.restype = C.c_int
        L.dq_max_d_in.restype = i32
        L.dq_quantize.restype = st
        L.dq_quantize.argtypes = [P, i32, i32, P, P, P, P]
        L.dq_build_colmajor.restype = st
        L.dq_build_colmajor.argtypes = [P, i32, i32, P, P]
        L.dq_split_gemv.restype = st
        L.dq_split_gemv.argtypes = [C.POINTER(DqWeights), P, P, f32, P, C.c_size_t, P]
        L.dq_split_gemv_noalloc.restype = st
        L.dq_split_gemv_noalloc.argtypes = [C.POINTER(DqWeights), P, P, f32, P]
        L.dq_reset_noalloc_workspace.restype = st
        L.dq_reset_noalloc_workspace.argtypes = [P]
        L.dq_split_gemv_batched.restype = st
        L.dq_split_gemv_batched.argtypes = [C.POINTER(DqWeights), P, P, i32, f32, P, C.c_size_t, P]
        L.dq_workspace_bytes_batched.restype = C.c_size_t
        L.dq_workspace_bytes_batched.argtypes = [i32, i32, i32]
        L.dq_split_gemv_batched_grouped.restype = st
        L.dq_split_gemv_batched_grouped.argtypes = [C.POINTER(DqWeights), C.POINTER(P), C.POINTER(P),
                                                    C.POINTER(i32), i32, f32, P, C.c_size_t, P]
        L.dq_workspace_bytes_batched_grouped.restype = C.c_size_t
        L.dq_workspace_bytes_batched_grouped.argtypes = [i32, i32, i32, i32]
        L.dq_silu_mul.restype = st
        L.dq_silu_mul.argtypes = [P, P, P, C.c_int64, P]
        L.dq_silu_mul_pairs.restype = st
        L.dq_silu_mul_pairs.argtypes = [P, P, i32, i32, P]
        L.dq_moe_combine.restype = st
        L.dq_moe_combine.argtypes = [P, P, P, P, i32, i32, P]
        L.dq_int4_gemv.restype = st
        L.dq_int4_gemv.argtypes = [C.POINTER(DqWeights), P, P, P, C.c_size_t, P]
        L.dq_workspace_bytes.restype = C.c_size_t
        L.dq_workspace_bytes.argtypes = [i32, i32]
        L.dq_reset_workspace.restype = st
        L.dq_reset_workspace.argtypes = [P, C.c_size_t, P]
        L.dq_reference_gemv.restype = st
        L.dq_reference_gemv.argtypes = [P, P, P, i32, i32, P]
        L.dq_detect_outliers.restype = st
        L.dq_detect_outliers.argtypes = [P, i32, f32, P, P, P, P, P]
        L.dq_native_bytes.restype = C.c_size_t
        L.dq_native_bytes.argtypes = [i32, i32]
        L.dq_build_native.restype = st
        L.dq_build_native.argtypes = [P, P, P, i32, i32, P, P]
        L.dq_read_device_error.restype = st
        L.dq_read_device_error.argtypes = [C.POINTER(C.c_uint32), C.c_int]
        L.dq_gather_region_bytes.restype = C.c_size_t
        L.dq_gather_region_bytes.argtypes = [i32]
        L.dq_split_gemv_gather.restype = st
        L.dq_split_gemv_gather.argtypes = [C.POINTER(DqWeights), P, P, f32, P, C.c_size_t, C.POINTER(DqGather), P]
        L.dq_device_alloc.restype = st
        L.dq_device_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)]
        L.dq_device_free.restype = st
        L.dq_device_free.argtypes = [P]
        L.dq_ipc_handle.restype = st
        L.dq_ipc_handle.argtypes = [P, C.c_char_p]
        L.dq_ipc_open.restype = st
        L.dq_ipc_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        L.dq_ipc_close.restype = st
        L.dq_ipc_close.argtypes = [P]
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().dq_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != DQ_OK:
        raise DqError(status, what, lib().dq_last_cuda_error() if status == DQ_ERR_CUDA else 0)


def batched_grouped(w_list, x_ptrs, y_ptrs, ms, k: float, ws_ptr: int, ws_bytes: int, stream: int) -> int:
    """dq_split_gemv_batched_grouped over len(w_list) problems (DqWeights,
    device addresses of x[e] and y[e], vector counts m[e]); returns the status."""
    n = len(w_list)
    w_arr = (DqWeights * n)(*w_list)
    x_arr = (C.c_void_p * n)(*x_ptrs)
    y_arr = (C.c_void_p * n)(*y_ptrs)
    m_arr = (C.c_int32 * n)(*ms)
    def vp(v):
        return v if isinstance(v, C.c_void_p) else C.c_void_p(v)
    return lib().dq_split_gemv_batched_grouped(w_arr, x_arr, y_arr, m_arr, n, float(k), vp(ws_ptr), ws_bytes,
                                               vp(stream))


def weights(packed: int, scales: int, zeros: int, fp16: int | None, fp16_cm: int | None,
            d_out: int, d_in: int, native: int | None = None) -> DqWeights:
    """Build a dq_weights_t from raw device addresses."""
    return DqWeights(packed, scales, zeros, fp16 or None, fp16_cm or None, native or None, d_out, d_in)
