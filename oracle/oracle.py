"""ctypes/numpy wrapper over oracle/liboracle.so (the C restatement in dq_oracle.c).

TEST INFRASTRUCTURE ONLY -- see oracle/__init__.py.

Arrays of binary16 values are numpy float16 (their bits are what the C side
reads); packed INT4 weights are uint8.  All functions take and return host
numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_QUANT = os.path.join(HERE, "_ref", "ref_quant")
REF_GPU_LIB = os.path.join(HERE, "_ref", "libdqref_gpu.so")

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import build_oracle
            build_oracle.build_liboracle()
        _lib = C.CDLL(LIB_PATH)
        P = C.c_void_p
        i, f = C.c_int, C.c_float
        _lib.dqo_h2f.restype = f
        _lib.dqo_h2f.argtypes = [C.c_uint16]
        _lib.dqo_f2h.restype = C.c_uint16
        _lib.dqo_f2h.argtypes = [f]
        _lib.dqo_h2f_array.argtypes = [P, P, C.c_int64]
        _lib.dqo_f2h_array.argtypes = [P, P, C.c_int64]
        _lib.dqo_quantize.restype = i
        _lib.dqo_quantize.argtypes = [P, i, i, P, P, P]
        _lib.dqo_detect.restype = i
        _lib.dqo_detect.argtypes = [P, i, f, P, P, P]
        _lib.dqo_split_gemv_masked.argtypes = [P, P, P, P, P, P, i, i, P, P]
        _lib.dqo_split_gemv.restype = i
        _lib.dqo_split_gemv.argtypes = [P, P, P, P, P, i, i, f, P, P, P]
        _lib.dqo_int4_gemv.argtypes = [P, P, P, P, i, i, P, P]
        _lib.dqo_reference_gemv.argtypes = [P, P, i, i, P, P]
        _lib.dqo_dense_gemv_f64.argtypes = [P, P, i, i, P]
        _lib.dqo_num_threads.restype = i
        _lib.dqo_set_num_threads.argtypes = [i]
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _h(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float16)


def f2h_bits(x: np.ndarray) -> np.ndarray:
    """binary32 -> binary16 (round to nearest even) via the C restatement."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.float16)
    lib().dqo_f2h_array(_p(x), _p(out), x.size)
    return out


def h2f(x: np.ndarray) -> np.ndarray:
    x = _h(x)
    out = np.empty(x.shape, dtype=np.float32)
    lib().dqo_h2f_array(_p(x), _p(out), x.size)
    return out


def quantize(w: np.ndarray):
    """src/quant_format.cuh:58-97 -> (packed u8 [d_out, d_in/2], scales f16 [d_out, G], zeros f16)."""
    w = _h(w)
    d_out, d_in = w.shape
    G = d_in // 128
    packed = np.empty((d_out, d_in // 2), dtype=np.uint8)
    scales = np.empty((d_out, G), dtype=np.float16)
    zeros = np.empty((d_out, G), dtype=np.float16)
    rc = lib().dqo_quantize(_p(w), d_out, d_in, _p(packed), _p(scales), _p(zeros))
    if rc:
        raise ValueError(f"bad shape {w.shape}")
    return packed, scales, zeros


def detect(x: np.ndarray, k: float):
    """src/outlier_detect.cuh:104-205 -> (mask u8 [d_in], indices int32 [count], stats f32 [4]).

    stats = (mean, thresh, var, M2).  indices are in the reference's list
    order (warp stripes in warp order, ascending inside each stripe)."""
    x = _h(x).reshape(-1)
    n = x.size
    mask = np.empty(n, dtype=np.uint8)
    idx = np.empty(max(n // 4, 1), dtype=np.int32)
    stats = np.empty(4, dtype=np.float32)
    c = lib().dqo_detect(_p(x), n, float(k), _p(mask), _p(idx), _p(stats))
    if c < 0:
        raise ValueError("bad input length")
    return mask, idx[:c].copy(), stats


def split_gemv(packed, scales, zeros, fp16_w, x, k: float = 3.0):
    """src/split_gemv.cu:75-158 -> (y16 f16 [d_out], y32 f32 [d_out], mask u8 [d_in])."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales, zeros, fp16_w, x = _h(scales), _h(zeros), _h(fp16_w), _h(x).reshape(-1)
    d_out, d_in = fp16_w.shape
    y32 = np.empty(d_out, dtype=np.float32)
    y16 = np.empty(d_out, dtype=np.float16)
    mask = np.empty(d_in, dtype=np.uint8)
    lib().dqo_split_gemv(_p(packed), _p(scales), _p(zeros), _p(fp16_w), _p(x), d_out, d_in,
                         float(k), _p(y32), _p(y16), _p(mask))
    return y16, y32, mask


def split_gemv_masked(packed, scales, zeros, fp16_w, x, mask):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales, zeros, fp16_w, x = _h(scales), _h(zeros), _h(fp16_w), _h(x).reshape(-1)
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    d_out, d_in = fp16_w.shape
    y32 = np.empty(d_out, dtype=np.float32)
    y16 = np.empty(d_out, dtype=np.float16)
    lib().dqo_split_gemv_masked(_p(packed), _p(scales), _p(zeros), _p(fp16_w), _p(x), _p(mask),
                                d_out, d_in, _p(y32), _p(y16))
    return y16, y32


def int4_gemv(packed, scales, zeros, x):
    """src/int4_gemv.cu:30-78 -> (y16, y32)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales, zeros, x = _h(scales), _h(zeros), _h(x).reshape(-1)
    d_out = packed.shape[0]
    d_in = packed.shape[1] * 2
    y32 = np.empty(d_out, dtype=np.float32)
    y16 = np.empty(d_out, dtype=np.float16)
    lib().dqo_int4_gemv(_p(packed), _p(scales), _p(zeros), _p(x), d_out, d_in, _p(y32), _p(y16))
    return y16, y32


def reference_gemv(w, x):
    """src/reference_gemv.cu:9-57 -> (y16, y32)."""
    w, x = _h(w), _h(x).reshape(-1)
    d_out, d_in = w.shape
    y32 = np.empty(d_out, dtype=np.float32)
    y16 = np.empty(d_out, dtype=np.float16)
    lib().dqo_reference_gemv(_p(w), _p(x), d_out, d_in, _p(y32), _p(y16))
    return y16, y32


def dense_gemv_f64(w, x) -> np.ndarray:
    """y = W x in binary64 over the FP16 inputs (accuracy yardstick)."""
    w, x = _h(w), _h(x).reshape(-1)
    d_out, d_in = w.shape
    y = np.empty(d_out, dtype=np.float64)
    lib().dqo_dense_gemv_f64(_p(w), _p(x), d_out, d_in, _p(y))
    return y


def num_threads() -> int:
    return lib().dqo_num_threads()


def set_num_threads(n: int) -> None:
    lib().dqo_set_num_threads(int(n))


def ref_quant_available() -> bool:
    return os.path.exists(REF_QUANT)


def ref_quantize(w: np.ndarray):
    """Run the reference's own host quantizer (oracle/_ref/ref_quant)."""
    w = _h(w)
    d_out, d_in = w.shape
    G = d_in // 128
    with tempfile.TemporaryDirectory() as td:
        wp = os.path.join(td, "w.f16")
        w.tofile(wp)
        pre = os.path.join(td, "q")
        subprocess.run([REF_QUANT, wp, str(d_out), str(d_in), pre], check=True)
        packed = np.fromfile(pre + ".packed", dtype=np.uint8).reshape(d_out, d_in // 2)
        scales = np.fromfile(pre + ".scales", dtype=np.float16).reshape(d_out, G)
        zeros = np.fromfile(pre + ".zeros", dtype=np.float16).reshape(d_out, G)
    return packed, scales, zeros
