"""GPU tests of the grouped batched split GEMV (dq_split_gemv_batched_grouped):
several problems of one shape, each with its own weights and its own 1-16
vectors, in one set of launches (the experts of a mixture-of-experts layer and
their routed tokens).  Every problem's rows must match the oracle's split GEMV
of each vector (src/split_gemv.cu:25-198 of dyn-quant applied per vector), and
equal the problem's own dq_split_gemv_batched call bit for bit when both run
the same vector-tile geometry (every m at most 8, or every m above 8)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dq_testutil import (  # noqa: E402
    abi, abi_build_native, abi_colmajor, abi_split_gemv_batched, abi_weights, check_y, dev, host, stream_ptr,
)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)


def _problems(d_out, d_in, ms, frac, layout, seed0=10):
    out = []
    for e, m in enumerate(ms):
        w = synth.weights(d_out, d_in, seed=seed0 + e)
        xs = synth.activations(m, d_in, frac, seed=seed0 + 50 + e)
        packed, scales, zeros = O.quantize(w)
        p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
        nat = abi_build_native(p_t, s_t, z_t)
        keep = [p_t, s_t, z_t, nat]
        if layout == "colmajor":
            cm = abi_colmajor(dev(w))
            keep.append(cm)
            wts = abi_weights(p_t, s_t, z_t, w_cm=cm, native=nat)
        else:
            rm = dev(w)
            keep.append(rm)
            wts = abi_weights(p_t, s_t, z_t, w_rm=rm, native=nat)
        out.append(dict(w=w, xs=xs, packed=packed, scales=scales, zeros=zeros, wts=wts, keep=keep, x_t=dev(xs)))
    return out


def _grouped(probs, k, ws=None):
    L = abi()
    d_out, d_in = probs[0]["wts"].d_out, probs[0]["wts"].d_in
    ms = [p["xs"].shape[0] for p in probs]
    need = L.lib().dq_workspace_bytes_batched_grouped(d_out, d_in, max(ms), len(probs))
    assert need > 0
    if ws is None:
        ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    ys = [torch.full((m, d_out), float("nan"), dtype=torch.float16, device="cuda") for m in ms]
    st = L.batched_grouped([p["wts"] for p in probs], [p["x_t"].data_ptr() for p in probs],
                           [y.data_ptr() for y in ys], ms, k, ws.data_ptr(), ws.numel(), stream_ptr())
    return st, ys


@pytest.mark.parametrize("d_out,d_in,ms,frac,layout", [
    (1024, 4096, [3, 8, 1, 5], 0.02, "colmajor"),     # one vector tile
    (2048, 8192, [16, 9, 12], 0.05, "colmajor"),      # two vector tiles
    (512, 28672, [2, 4, 6], 0.03, "colmajor"),        # longest rows
    (1000, 4096, [7, 2], 0.05, "colmajor"),           # ragged rows (direct outlier loads)
    (1024, 4096, [4, 4, 4, 4, 4, 4, 4, 4], 0.02, "rowmajor"),  # eight experts, row-major FP16 only
])
def test_grouped_equals_separate_calls(d_out, d_in, ms, frac, layout):
    probs = _problems(d_out, d_in, ms, frac, layout)
    st, ys = _grouped(probs, 3.0)
    assert st == 0, abi().status_string(st)
    torch.cuda.synchronize()
    for e, p in enumerate(probs):
        ref = host(abi_split_gemv_batched(p["wts"], p["x_t"], 3.0))
        got = host(ys[e])
        assert np.array_equal(got.view(np.int16), ref.view(np.int16)), f"problem {e}: not the separate call's result"


def test_grouped_mixed_tiles_match_the_oracle():
    """m = 16 beside m = 3: the small problem runs in the two-tile geometry."""
    probs = _problems(1024, 8192, [16, 3, 9], 0.05, "colmajor", seed0=30)
    st, ys = _grouped(probs, 3.0)
    assert st == 0
    torch.cuda.synchronize()
    for e, p in enumerate(probs):
        y = host(ys[e])
        for i, x in enumerate(p["xs"]):
            y16, y32, _ = O.split_gemv(p["packed"], p["scales"], p["zeros"], p["w"], x, 3.0)
            check_y(y[i], y16, y32, what=f"problem {e} row {i}")
        ref = host(abi_split_gemv_batched(p["wts"], p["x_t"], 3.0))
        check_y(y, ref, None, what=f"problem {e} vs its separate call")


def test_grouped_repeats_bit_for_bit():
    probs = _problems(2048, 4096, [5, 2, 8], 0.02, "colmajor", seed0=40)
    st, ys1 = _grouped(probs, 3.0)
    assert st == 0
    st, ys2 = _grouped(probs, 3.0)
    assert st == 0
    torch.cuda.synchronize()
    for a, b in zip(ys1, ys2):
        assert np.array_equal(host(a).view(np.int16), host(b).view(np.int16))


def test_grouped_rejects_bad_arguments():
    L = abi()
    probs = _problems(256, 1024, [2, 3], 0.02, "colmajor", seed0=50)
    ws = torch.zeros(L.lib().dq_workspace_bytes_batched_grouped(256, 1024, 3, 2), dtype=torch.uint8, device="cuda")
    y = torch.empty((3, 256), dtype=torch.float16, device="cuda")
    w = [p["wts"] for p in probs]
    x = [p["x_t"].data_ptr() for p in probs]

    def call(ws_, ms, ww=w, xx=x, n=None):
        return L.batched_grouped(ww[:n] if n else ww, xx[:n] if n else xx, [y.data_ptr()] * len(ms), ms, 3.0,
                                 ws_.data_ptr(), ws_.numel(), stream_ptr())
    assert call(ws, [2, 0]) == 2                     # m = 0
    assert call(ws, [2, 17]) == 2                    # m > 16
    small = ws[: ws.numel() // 2]
    assert call(small, [2, 3]) == 6                  # workspace too small
    other = _problems(256, 2048, [2], 0.02, "colmajor", seed0=60)
    assert call(ws, [2, 2], ww=[w[0], other[0]["wts"]], xx=[x[0], other[0]["x_t"].data_ptr()]) == 2  # shapes differ
    assert L.lib().dq_workspace_bytes_batched_grouped(256, 1024, 3, 17) == 0
    assert L.lib().dq_workspace_bytes_batched_grouped(256, 1024, 0, 2) == 0
    err = C.c_uint32(0)
    assert L.lib().dq_read_device_error(C.byref(err), 0) == 0
