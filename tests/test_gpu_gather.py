"""The split GEMV with the row-sharded gather fused (dq_split_gemv_gather), on
one GPU.

* world 1: the gathered call is the plain split GEMV, bit for bit, call after
  call (the two slices of the region alternate).
* rank 0 of 2: the other rank is emulated from the host, which plants that
  rank's published rows in its region and its flags in rank 0's region before
  each call; rank 0's kernel must return its own rows, the planted rows in
  the other rank's place, and raise its own flags in the other region.  No
  second kernel runs: nothing on this GPU waits for another kernel.
* the bounded wait running out: no flags planted, so the wait gives up after
  about a second; the kernel reports bit 4 of the device error word, writes
  its own rows and leaves the other rank's rows untouched.

Region layout (include/dq_abi.h, dq_gather_t): two slices of rows_per FP16
rows (each padded to 256 bytes), flags [8][1024] u32, epoch [1024] u32.
"""
import ctypes as C

import numpy as np
import pytest

from dq_testutil import (_ptr, abi, abi_build_native, abi_colmajor, abi_quantize, abi_split_gemv, abi_weights,
                         dev, host, stream_ptr, workspace)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_CTAS = 1024
MAX_RANKS = 8


def _layout(rows_per):
    slice_b = (rows_per * 2 + 255) // 256 * 256
    flags = 2 * slice_b
    epoch = flags + MAX_RANKS * MAX_CTAS * 4
    total = (epoch + MAX_CTAS * 4 + 255) // 256 * 256
    return slice_b, flags, epoch, total


def _weights(d_out, d_in, seed):
    from dyn_quant import synth
    w = torch.from_numpy(synth.weights(d_out, d_in, seed=seed)).cuda()
    packed, scales, zeros = abi_quantize(w)
    return abi_weights(packed, scales, zeros, w_cm=abi_colmajor(w), native=abi_build_native(packed, scales, zeros))


def _gather(wts, x, y, g):
    _lib = abi()
    ws = workspace(wts.d_out, wts.d_in)
    return _lib.lib().dq_split_gemv_gather(C.byref(wts), _ptr(x), _ptr(y), 3.0, _ptr(ws), ws.numel(), C.byref(g),
                                           stream_ptr())


def _desc(rank, world, rows_per, d_total, regions):
    _lib = abi()
    arr = (C.c_void_p * MAX_RANKS)(*([r.data_ptr() for r in regions] + [None] * (MAX_RANKS - len(regions))))
    return _lib.DqGather(rank, world, rows_per, d_total, arr)


def _u32(region, off, n):
    return region[off:off + 4 * n].view(torch.int32)


def test_region_bytes():
    L = abi().lib()
    for rows in (16, 1024, 3584, 11008):
        assert L.dq_gather_region_bytes(rows) == _layout(rows)[3]
    assert L.dq_gather_region_bytes(0) == 0 and L.dq_gather_region_bytes(100) == 0


def test_world_one_is_the_split_gemv():
    from dyn_quant import synth
    rows_per, d_in = 1024, 4096
    wts = _weights(rows_per, d_in, seed=3)
    region = torch.zeros(_layout(rows_per)[3], dtype=torch.uint8, device="cuda")
    g = _desc(0, 1, rows_per, rows_per, [region])
    for call in range(1, 4):
        x = dev(synth.activation(d_in, 0.02, seed=30 + call))
        y = torch.empty(rows_per, dtype=torch.float16, device="cuda")
        assert _gather(wts, x, y, g) == 0
        ref = abi_split_gemv(wts, x, 3.0)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), f"call {call}"
        epoch = host(_u32(region, _layout(rows_per)[2], MAX_CTAS))
        grid = int((epoch > 0).sum())
        assert grid > 0 and (epoch[:grid] == call).all() and (epoch[grid:] == 0).all()


@pytest.mark.parametrize("rows_per,d_in,tail", [(1024, 4096, 5), (3584, 8192, 0), (512, 11008, 16)])
def test_rank0_of_two_with_planted_peer(rows_per, d_in, tail):
    from dyn_quant import synth
    slice_b, flags_off, epoch_off, total = _layout(rows_per)
    d_total = 2 * rows_per - tail
    wts = _weights(rows_per, d_in, seed=4)
    r0 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    r1 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    g = _desc(0, 2, rows_per, d_total, [r0, r1])
    rng = np.random.default_rng(5)
    for call in range(1, 4):
        x = dev(synth.activation(d_in, 0.02, seed=40 + call))
        # rank 1 has published call `call`: its rows in its slice, its flags in rank 0's region
        peer_rows = rng.standard_normal(rows_per).astype(np.float16)
        par = call & 1
        r1[par * slice_b:par * slice_b + 2 * rows_per].view(torch.float16).copy_(dev(peer_rows))
        _u32(r0, flags_off + 1 * MAX_CTAS * 4, MAX_CTAS).fill_(call)
        y = torch.full((d_total,), float("nan"), dtype=torch.float16, device="cuda")
        assert _gather(wts, x, y, g) == 0
        own = abi_split_gemv(wts, x, 3.0)
        torch.cuda.synchronize()
        yh = host(y)
        assert np.array_equal(yh[:rows_per].view(np.int16), host(own).view(np.int16)), f"call {call}: own rows"
        assert np.array_equal(yh[rows_per:].view(np.int16), peer_rows[:d_total - rows_per].view(np.int16)), \
            f"call {call}: the other rank's rows"
        # rank 0 published in its own slice and raised its flags in rank 1's region
        mine = host(r0[par * slice_b:par * slice_b + 2 * rows_per].view(torch.float16))
        assert np.array_equal(mine.view(np.int16), host(own).view(np.int16))
        epoch = host(_u32(r0, epoch_off, MAX_CTAS))
        grid = int((epoch > 0).sum())
        raised = host(_u32(r1, flags_off + 0 * MAX_CTAS * 4, MAX_CTAS))
        assert (epoch[:grid] == call).all() and (raised[:grid] == call).all() and (raised[grid:] == 0).all()
    err = C.c_uint32(0)
    assert abi().lib().dq_read_device_error(C.byref(err), 0) == 0 and err.value & 16 == 0


def test_wait_runs_out():
    """No flags from the other rank: the bounded wait gives up (about a second)."""
    from dyn_quant import synth
    _lib = abi()
    rows_per, d_in = 256, 4096
    _, _, _, total = _layout(rows_per)
    wts = _weights(rows_per, d_in, seed=6)
    r0 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    r1 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    g = _desc(0, 2, rows_per, 2 * rows_per, [r0, r1])
    x = dev(synth.activation(d_in, 0.02, seed=7))
    y = torch.full((2 * rows_per,), 7.0, dtype=torch.float16, device="cuda")
    err = C.c_uint32(0)
    assert _lib.lib().dq_read_device_error(C.byref(err), 1) == 0
    assert _gather(wts, x, y, g) == 0
    own = abi_split_gemv(wts, x, 3.0)
    torch.cuda.synchronize()
    assert _lib.lib().dq_read_device_error(C.byref(err), 1) == 0
    assert err.value & 16, f"error word {err.value:#x}: the wait should have run out"
    yh = host(y)
    assert np.array_equal(yh[:rows_per].view(np.int16), host(own).view(np.int16))
    assert (yh[rows_per:] == 7.0).all()


def test_bad_arguments():
    _lib = abi()
    L = _lib.lib()
    rows_per, d_in = 256, 4096
    wts = _weights(rows_per, d_in, seed=8)
    region = torch.zeros(_layout(rows_per)[3], dtype=torch.uint8, device="cuda")
    x = torch.zeros(d_in, dtype=torch.float16, device="cuda")
    y = torch.zeros(rows_per, dtype=torch.float16, device="cuda")
    ws = workspace(rows_per, d_in)

    def call(g, w=wts):
        return L.dq_split_gemv_gather(C.byref(w), _ptr(x), _ptr(y), 3.0, _ptr(ws), ws.numel(), C.byref(g),
                                      stream_ptr())
    assert call(_desc(0, 1, rows_per, rows_per, [region])) == 0
    assert call(_desc(1, 1, rows_per, rows_per, [region])) == _lib.DQ_ERR_INVALID_ARGUMENT  # rank >= world
    assert call(_desc(0, 9, rows_per, rows_per, [region] * 8)) == _lib.DQ_ERR_INVALID_ARGUMENT
    assert call(_desc(0, 1, 2 * rows_per, 2 * rows_per, [region])) == _lib.DQ_ERR_SHAPE  # d_out != rows_per
    assert call(_desc(0, 1, rows_per, rows_per + 1, [region])) == _lib.DQ_ERR_SHAPE
    assert call(_desc(0, 2, rows_per, rows_per, [region, region])) == _lib.DQ_ERR_SHAPE  # d_total too small
    g = _desc(0, 2, rows_per, 2 * rows_per, [region])  # region[1] missing
    assert call(g) == _lib.DQ_ERR_INVALID_ARGUMENT
    no_native = abi_weights(*wts._keep[:3], w_cm=wts._keep[4])
    assert call(_desc(0, 1, rows_per, rows_per, [region]), no_native) == _lib.DQ_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
