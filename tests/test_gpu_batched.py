"""GPU parity of the batched split GEMV (dq_split_gemv_batched, 1 <= m <= 16
vectors per call) against the oracle: every row of the batch is the oracle's
batch-1 split GEMV of that vector, with that vector's own outlier mask
(src/split_gemv.cu:25-198 of dyn-quant applied per vector)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dq_testutil import (  # noqa: E402
    abi, abi_build_native, abi_colmajor, abi_detect, abi_split_gemv, abi_split_gemv_batched, abi_weights, check_y,
    dev, host,
)

# (d_out, d_in, outlier fraction, k, distribution, m)
CASES = [
    (4096, 4096, 0.02, 3.0, "normal", 4),     # 7B q_proj, the sweep's batch sizes
    (4096, 4096, 0.02, 3.0, "normal", 16),
    (11008, 4096, 0.01, 3.0, "normal", 8),    # 7B gate
    (1024, 11008, 0.01, 3.0, "normal", 5),    # 7B down width, partial last chunk
    (2048, 8192, 0.05, 3.0, "normal", 9),     # sweep width, 5 % outliers, two vector tiles
    (2048, 8192, 0.0, 4.0, "normal", 16),     # no outliers at all
    (1024, 8192, 0.05, 2.0, "t3", 7),         # heavy tails, low k: a large union
    (512, 28672, 0.03, 3.0, "normal", 3),     # 70B down width
    (100, 256, 0.05, 3.0, "normal", 16),      # ragged rows (direct outlier loads)
    (37, 1152, 0.10, 2.0, "normal", 2),       # ragged rows, many outliers
    (1, 128, 0.05, 2.0, "normal", 1),         # smallest
    (1024, 4096, 0.10, 1.0, "normal", 12),    # most channels outliers: capacity rule per vector
    (8192, 8192, 0.05, 3.0, "normal", 16),    # the sweep's full 8192 x 8192 shape at its largest batch
]
IDS = [f"{a}x{b}-f{c}-k{d}-{e}-m{f}" for a, b, c, d, e, f in CASES]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)


def _case(d_out, d_in, frac, dist, m, seed=0):
    w = synth.weights(d_out, d_in, seed=seed)
    xs = synth.activations(m, d_in, frac, seed=1 + 100 * seed, dist=dist)
    packed, scales, zeros = O.quantize(w)
    return w, xs, packed, scales, zeros


def _weights(w, packed, scales, zeros, layout):
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    nat = abi_build_native(p_t, s_t, z_t)
    if layout == "colmajor":
        return abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(dev(w)), native=nat)
    return abi_weights(p_t, s_t, z_t, w_rm=dev(w), native=nat)


def _check_rows(y, w, xs, packed, scales, zeros, k):
    for i, x in enumerate(xs):
        gmask, _, _ = abi_detect(dev(x), k)
        y16m, y32m = O.split_gemv_masked(packed, scales, zeros, w, x, gmask.astype(np.uint8))
        check_y(y[i], y16m, y32m, what=f"row {i} (gpu mask)")
        y16, _, _ = O.split_gemv(packed, scales, zeros, w, x, k)
        check_y(y[i], y16, None, what=f"row {i} (oracle mask)")


@pytest.mark.parametrize("layout", ["colmajor", "rowmajor"])
@pytest.mark.parametrize("d_out,d_in,frac,k,dist,m", CASES, ids=IDS)
def test_batched_matches_oracle(d_out, d_in, frac, k, dist, m, layout):
    w, xs, packed, scales, zeros = _case(d_out, d_in, frac, dist, m)
    wts = _weights(w, packed, scales, zeros, layout)
    y = host(abi_split_gemv_batched(wts, dev(xs), k))
    assert y.shape == (m, d_out)
    _check_rows(y, w, xs, packed, scales, zeros, k)


def test_batched_is_reproducible_and_shares_the_workspace():
    """Fixed summation order: repeated calls are bit-identical; batch-1 and
    batched calls alternate on one zero-filled workspace."""
    d_out, d_in, k = 2048, 8192, 3.0
    w, xs, packed, scales, zeros = _case(d_out, d_in, 0.03, "normal", 11, seed=2)
    wts = _weights(w, packed, scales, zeros, "colmajor")
    L = abi().lib()
    need = max(L.dq_workspace_bytes_batched(d_out, d_in, 11), L.dq_workspace_bytes(d_out, d_in))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    x_t = dev(xs)
    ys = []
    for _ in range(3):
        ys.append(host(abi_split_gemv_batched(wts, x_t, k, ws=ws)))
        y1 = torch.empty(d_out, dtype=torch.float16, device="cuda")
        import ctypes as C
        abi().check(L.dq_split_gemv(C.byref(wts), C.c_void_p(x_t[3].data_ptr()), C.c_void_p(y1.data_ptr()),
                                    k, C.c_void_p(ws.data_ptr()), ws.numel(),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream)), "dq_split_gemv")
        y16, _, _ = O.split_gemv(packed, scales, zeros, w, xs[3], k)
        check_y(host(y1), y16, None, what="batch-1 between batched calls")
    assert all(np.array_equal(ys[0].view(np.uint16), y.view(np.uint16)) for y in ys[1:])
    _check_rows(ys[0], w, xs, packed, scales, zeros, k)


def test_batched_rows_agree_with_batch1():
    d_out, d_in, k = 4096, 4096, 3.0
    w, xs, packed, scales, zeros = _case(d_out, d_in, 0.02, "normal", 6, seed=3)
    wts = _weights(w, packed, scales, zeros, "colmajor")
    y = host(abi_split_gemv_batched(wts, dev(xs), k))
    for i, x in enumerate(xs):
        y1 = host(abi_split_gemv(wts, dev(x), k))
        check_y(y[i], y1, None, what=f"row {i} vs batch-1")


def test_python_api_batches():
    """DynQuantLinear.forward on [m, d_in]: rows through the batched kernel
    (more than 16 rows: several calls); [d_in] and [1, d_in] keep the
    reference's batch-1 result shape."""
    import dyn_quant
    d_out, d_in, k = 1024, 4096, 3.0
    w, xs, packed, scales, zeros = _case(d_out, d_in, 0.02, "normal", 20, seed=4)
    lin = dyn_quant.DynQuantLinear(d_in, d_out, k)
    lin.load_weight(dev(w))
    y = host(lin(dev(xs)))
    assert y.shape == (20, d_out)
    _check_rows(y, w, xs, packed, scales, zeros, k)
    assert tuple(lin(dev(xs[0])).shape) == (d_out,)
    assert tuple(lin(dev(xs[:1])).shape) == (d_out,)
    assert tuple(lin(dev(xs[:0].reshape(0, d_in))).shape) == (0, d_out)


def test_batched_rejects_bad_arguments():
    import ctypes as C
    L = abi().lib()
    d_out, d_in = 64, 256
    w, xs, packed, scales, zeros = _case(d_out, d_in, 0.02, "normal", 2)
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    x_t = dev(xs)
    y = torch.empty((17, d_out), dtype=torch.float16, device="cuda")
    ws = torch.zeros(L.dq_workspace_bytes_batched(d_out, d_in, 16), dtype=torch.uint8, device="cuda")
    no_native = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(dev(w)))
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (C.c_void_p(x_t.data_ptr()), C.c_void_p(y.data_ptr()))
    assert L.dq_split_gemv_batched(C.byref(no_native), *args, 2, 3.0, C.c_void_p(ws.data_ptr()), ws.numel(), sp) == 1
    wts = _weights(w, packed, scales, zeros, "colmajor")
    assert L.dq_split_gemv_batched(C.byref(wts), *args, 0, 3.0, C.c_void_p(ws.data_ptr()), ws.numel(), sp) == 2
    assert L.dq_split_gemv_batched(C.byref(wts), *args, 17, 3.0, C.c_void_p(ws.data_ptr()), ws.numel(), sp) == 2
    assert L.dq_split_gemv_batched(C.byref(wts), *args, 2, 3.0, C.c_void_p(ws.data_ptr()), 1024, sp) == 6
    assert L.dq_workspace_bytes_batched(d_out, d_in, 17) == 0
