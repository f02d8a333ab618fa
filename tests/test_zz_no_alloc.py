"""dq_split_gemv_noalloc (the split GEMV whose workspace is the library's static
device array) against dq_split_gemv with a caller workspace and against the
oracle: same inputs, two calls in a row, through the C ABI.  Also checks that
the entry point allocates no device memory."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dq_testutil import (  # noqa: E402
    abi, abi_build_native, abi_colmajor, abi_split_gemv, abi_weights, check_y, dev, host, stream_ptr,
)


def noalloc_into(wts, x_t, y, k):
    _lib = abi()
    _lib.check(_lib.lib().dq_split_gemv_noalloc(C.byref(wts), C.c_void_p(x_t.data_ptr()), C.c_void_p(y.data_ptr()),
                                                float(k), stream_ptr()), "dq_split_gemv_noalloc")
    return y


def noalloc_split_gemv(wts, x_t, k):
    return noalloc_into(wts, x_t, torch.empty(wts.d_out, dtype=torch.float16, device=x_t.device), k)


def _weights(w, layout):
    packed, scales, zeros = O.quantize(w)
    p_t, s_t, z_t, w_t = dev(packed), dev(scales), dev(zeros), dev(w)
    nat = abi_build_native(p_t, s_t, z_t) if layout.endswith("native") else None
    if layout.startswith("colmajor"):
        wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(w_t), native=nat)
    else:
        wts = abi_weights(p_t, s_t, z_t, w_rm=w_t, native=nat)
    return wts, packed, scales, zeros


@pytest.mark.parametrize("d_out,d_in,frac,layout", [
    (4096, 4096, 0.02, "colmajor+native"),
    (11008, 4096, 0.01, "colmajor+native"),
    (1024, 11008, 0.03, "colmajor"),
    (100, 256, 0.05, "rowmajor"),
])
def test_noalloc_matches_workspace_entry_point(d_out, d_in, frac, layout):
    torch.cuda.set_device(0)
    w = synth.weights(d_out, d_in, seed=0)
    wts, packed, scales, zeros = _weights(w, layout)
    for call in range(2):
        x = synth.activation(d_in, frac, seed=10 + call)
        x_t = dev(x)
        ref = host(abi_split_gemv(wts, x_t, 3.0))
        got = host(noalloc_split_gemv(wts, x_t, 3.0))
        check_y(got, ref, what=f"noalloc call {call + 1} vs dq_split_gemv")
        y16, _, _ = O.split_gemv(packed, scales, zeros, w, x, 3.0)
        check_y(got, y16, what=f"noalloc call {call + 1} vs the oracle")
    word = C.c_uint32(0)
    abi().check(abi().lib().dq_read_device_error(C.byref(word), 1), "dq_read_device_error")
    assert word.value == 0


def test_noalloc_allocates_no_device_memory():
    """After the first call (which looks up the static array), further calls
    with preallocated x and y leave the device's free memory unchanged."""
    torch.cuda.set_device(0)
    d_out, d_in = 2048, 4096
    w = synth.weights(d_out, d_in, seed=3)
    wts, _, _, _ = _weights(w, "colmajor+native")
    x_t = dev(synth.activation(d_in, 0.02, seed=4))
    y = torch.empty(d_out, dtype=torch.float16, device="cuda")
    noalloc_into(wts, x_t, y, 3.0)
    torch.cuda.synchronize()
    first = host(y).copy()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(8):
        noalloc_into(wts, x_t, y, 3.0)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    assert np.array_equal(host(y).view(np.uint16), first.view(np.uint16))  # bit-reproducible


def test_noalloc_reset_keeps_results():
    """dq_reset_noalloc_workspace zeroes the static array on a stream; calls
    before and after it give the same bits."""
    torch.cuda.set_device(0)
    d_out, d_in = 1024, 8192
    w = synth.weights(d_out, d_in, seed=7)
    wts, _, _, _ = _weights(w, "colmajor+native")
    x_t = dev(synth.activation(d_in, 0.03, seed=8))
    y0 = host(noalloc_split_gemv(wts, x_t, 3.0)).copy()
    _lib = abi()
    _lib.check(_lib.lib().dq_reset_noalloc_workspace(stream_ptr()), "dq_reset_noalloc_workspace")
    y1 = host(noalloc_split_gemv(wts, x_t, 3.0))
    assert np.array_equal(y0.view(np.uint16), y1.view(np.uint16))


def test_noalloc_rejects_bad_arguments():
    _lib = abi()
    L = _lib.lib()
    w = _lib.weights(16, 16, 16, None, None, 16, 128)
    assert L.dq_split_gemv_noalloc(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, None) == _lib.DQ_ERR_INVALID_ARGUMENT
    w = _lib.weights(16, 16, 16, 16, None, 16, 100)
    assert L.dq_split_gemv_noalloc(C.byref(w), C.c_void_p(16), C.c_void_p(16), 3.0, None) == _lib.DQ_ERR_SHAPE
    assert L.dq_split_gemv_noalloc(None, C.c_void_p(16), C.c_void_p(16), 3.0, None) == _lib.DQ_ERR_INVALID_ARGUMENT
