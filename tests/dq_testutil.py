"""Shared helpers for the parity tests: C-ABI calls on torch device buffers and
the tolerance rules.

Tolerances (FP16 output y of a GEMV against the oracle's FP16/FP32 output):
  * rel-L2(y, y_ref16)  <= 1e-3
  * |y - y_ref16|       <= max(1e-2, one FP16 ulp of y_ref16): two FP32 sums that
    differ in the last bits can round to neighbouring FP16 values, and for
    |y| >= 16 one FP16 ulp (2^-6) is larger than 1e-2
  * |y - y_ref32|       <= half an FP16 ulp of y_ref32 + 1e-3 (y is the FP16
    rounding of an FP32 sum that agrees with the oracle's to ~1e-4)
Outlier mask: identical except channels within 1e-5 relative of the threshold.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

MAX_ABS = 1e-2
REL_L2 = 1e-3
MASK_BAND = 1e-5


def f16_ulp(v: np.ndarray) -> np.ndarray:
    a = np.abs(np.asarray(v, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


def check_y(y16: np.ndarray, ref16: np.ndarray, ref32: np.ndarray | None = None, what: str = "y",
            rows: np.ndarray | None = None) -> dict:
    y = np.asarray(y16, dtype=np.float64)
    r = np.asarray(ref16, dtype=np.float64)
    if rows is not None:
        y, r = y[rows], r[rows]
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    err = np.abs(y - r)
    tol = np.maximum(MAX_ABS, f16_ulp(r))
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, (f"{what}: {bad.size} outputs outside max(1e-2, 1 ulp); first {bad[:5]} "
                           f"y={y[bad[:5]]} ref={r[bad[:5]]}")
    rl = rel_l2(y, r)
    assert rl <= REL_L2, f"{what}: rel-L2 {rl:.3e} > {REL_L2}"
    out = {"max_abs": float(err.max()) if err.size else 0.0, "rel_l2": rl}
    if ref32 is not None:
        r32 = np.asarray(ref32, dtype=np.float64)
        if rows is not None:
            r32 = r32[rows]
        e32 = np.abs(y - r32)
        tol32 = 0.5 * f16_ulp(r32) + 1e-3
        bad = np.nonzero(e32 > tol32)[0]
        assert bad.size == 0, (f"{what}: {bad.size} outputs not the FP16 rounding of the oracle FP32 sum; "
                               f"first {bad[:5]} y={y[bad[:5]]} ref32={r32[bad[:5]]}")
        out["max_abs_vs_f32"] = float(e32.max()) if e32.size else 0.0
    return out


def check_mask(mask: np.ndarray, ref_mask: np.ndarray, x: np.ndarray, mean: float, thresh: float,
               what: str = "mask") -> int:
    """Returns the number of differing channels (all within the 1e-5 band)."""
    m = np.asarray(mask).astype(bool)
    r = np.asarray(ref_mask).astype(bool)
    diff = np.nonzero(m != r)[0]
    if diff.size:
        xf = np.asarray(x, dtype=np.float64)
        margin = np.abs(np.abs(xf[diff] - mean) - thresh)
        far = diff[margin > MASK_BAND * abs(thresh)]
        assert far.size == 0, f"{what}: channels {far[:8]} differ away from the threshold"
    return int(diff.size)


# ---------------------------------------------------------------------------
# C-ABI on torch device buffers
# ---------------------------------------------------------------------------
def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_ptr():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def abi():
    from dyn_quant import _lib
    return _lib


def dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t) -> np.ndarray:
    return t.detach().cpu().numpy()


def abi_quantize(w_t):
    import torch
    _lib = abi()
    d_out, d_in = w_t.shape
    packed = torch.empty((d_out, d_in // 2), dtype=torch.uint8, device=w_t.device)
    scales = torch.empty((d_out, d_in // 128), dtype=torch.float16, device=w_t.device)
    zeros = torch.empty_like(scales)
    _lib.check(_lib.lib().dq_quantize(_ptr(w_t), d_out, d_in, _ptr(packed), _ptr(scales), _ptr(zeros),
                                      stream_ptr()), "dq_quantize")
    return packed, scales, zeros


def abi_colmajor(w_t):
    import torch
    _lib = abi()
    d_out, d_in = w_t.shape
    cm = torch.empty((d_in, d_out), dtype=torch.float16, device=w_t.device)
    _lib.check(_lib.lib().dq_build_colmajor(_ptr(w_t), d_out, d_in, _ptr(cm), stream_ptr()),
               "dq_build_colmajor")
    return cm


def abi_build_native(packed, scales, zeros):
    import torch
    _lib = abi()
    d_out, half = packed.shape
    n = _lib.lib().dq_native_bytes(d_out, half * 2)
    out = torch.empty(n, dtype=torch.uint8, device=packed.device)
    _lib.check(_lib.lib().dq_build_native(_ptr(packed), _ptr(scales), _ptr(zeros), d_out, half * 2, _ptr(out),
                                          stream_ptr()), "dq_build_native")
    return out


def abi_weights(packed, scales, zeros, w_rm=None, w_cm=None, native=None):
    _lib = abi()
    d_out, half = packed.shape
    w = _lib.weights(packed.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                     None if w_rm is None else w_rm.data_ptr(),
                     None if w_cm is None else w_cm.data_ptr(), d_out, half * 2,
                     None if native is None else native.data_ptr())
    w._keep = (packed, scales, zeros, w_rm, w_cm, native)  # keep the buffers alive with the view
    return w


_workspaces = {}


def workspace(d_out: int, d_in: int, device=None):
    """A zero-filled GEMV workspace for the current stream, grown on demand."""
    import torch
    _lib = abi()
    need = _lib.lib().dq_workspace_bytes(d_out, d_in)
    key = (torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device="cuda")
        _workspaces[key] = ws
    return ws


def abi_split_gemv(wts, x_t, k: float):
    import torch
    _lib = abi()
    y = torch.empty(wts.d_out, dtype=torch.float16, device=x_t.device)
    ws = workspace(wts.d_out, wts.d_in)
    _lib.check(_lib.lib().dq_split_gemv(C.byref(wts), _ptr(x_t), _ptr(y), float(k), _ptr(ws), ws.numel(),
                                        stream_ptr()), "dq_split_gemv")
    return y


def abi_split_gemv_batched(wts, x_t, k: float, ws=None):
    """x_t [m, d_in] -> y [m, d_out] through dq_split_gemv_batched."""
    import torch
    _lib = abi()
    m = x_t.shape[0]
    y = torch.empty((m, wts.d_out), dtype=torch.float16, device=x_t.device)
    if ws is None:
        need = _lib.lib().dq_workspace_bytes_batched(wts.d_out, wts.d_in, m)
        key = ("batched", torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device="cuda")
            _workspaces[key] = ws
    _lib.check(_lib.lib().dq_split_gemv_batched(C.byref(wts), _ptr(x_t), _ptr(y), m, float(k), _ptr(ws), ws.numel(),
                                                stream_ptr()), "dq_split_gemv_batched")
    return y


def abi_int4_gemv(wts, x_t):
    import torch
    _lib = abi()
    y = torch.empty(wts.d_out, dtype=torch.float16, device=x_t.device)
    ws = workspace(wts.d_out, wts.d_in)
    _lib.check(_lib.lib().dq_int4_gemv(C.byref(wts), _ptr(x_t), _ptr(y), _ptr(ws), ws.numel(), stream_ptr()),
               "dq_int4_gemv")
    return y


def abi_reference_gemv(w_t, x_t):
    import torch
    _lib = abi()
    d_out, d_in = w_t.shape
    y = torch.empty(d_out, dtype=torch.float16, device=x_t.device)
    _lib.check(_lib.lib().dq_reference_gemv(_ptr(w_t), _ptr(x_t), _ptr(y), d_out, d_in, stream_ptr()),
               "dq_reference_gemv")
    return y


def abi_detect(x_t, k: float):
    """-> (mask bool [d_in], indices int32 [count], stats f32 [4]) as numpy."""
    import torch
    _lib = abi()
    d_in = x_t.numel()
    words = torch.empty(d_in // 32, dtype=torch.int32, device=x_t.device)
    idx = torch.empty(max(d_in // 4, 1), dtype=torch.int32, device=x_t.device)
    cnt = torch.empty(1, dtype=torch.int32, device=x_t.device)
    stats = torch.empty(4, dtype=torch.float32, device=x_t.device)
    _lib.check(_lib.lib().dq_detect_outliers(_ptr(x_t), d_in, float(k), _ptr(words), _ptr(idx), _ptr(cnt),
                                             _ptr(stats), stream_ptr()), "dq_detect_outliers")
    w = host(words).view(np.uint32)
    mask = ((w[:, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(-1).astype(bool)
    n = int(host(cnt)[0])
    return mask, host(idx)[:n], host(stats)
