"""The split GEMV with the row-sharded gather fused (dq_split_gemv_gather), on
one GPU.

* world 1: the gathered call agrees with the plain split GEMV and the
  oracle, and repeats itself bit for bit.
* rank 0 of 2: the other rank is emulated from the host, which plants that
  rank's rows in rank 0's region (the copy of the call's parity) as tagged
  words before each call.  Rank 0's kernel must return its own rows and the
  planted rows in the other rank's place, and store its own rows, tagged,
  in the other region's copy.  No second kernel runs: nothing on this GPU
  waits for another kernel.
* the bounded wait running out: nothing planted, so the waits give up
  after about a second; the kernel reports bit 4 of the device error word,
  writes its own rows and leaves the other rank's rows untouched.

Region layout (include/dq_abi.h, dq_split_gemv_gather): a 256-byte header
(u32 calls completed), then two copies of the full output (8 x rows_per
32-bit words, padded to 256 bytes) for calls of parity 0 and 1; a word is
the FP16 value | the low 16 bits of the call's number << 16.
"""
import ctypes as C

import numpy as np
import pytest

from dq_testutil import _ptr, abi, abi_build_native, abi_colmajor, abi_quantize, abi_split_gemv, abi_weights, check_y, \
    dev, host, stream_ptr, workspace

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_RANKS = 8


def _layout(rows_per):
    ybytes = (MAX_RANKS * rows_per * 4 + 255) // 256 * 256
    return 256, ybytes, 256 + 2 * ybytes  # copies start, bytes per copy, total


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


def _hdr(region):
    return host(region[:4].view(torch.int32))


def _words(region, rows_per, par, n):
    """The first n words of the region's copy of parity par (int32 view)."""
    start, ybytes, _ = _layout(rows_per)
    return region[start + par * ybytes:start + par * ybytes + 4 * n].view(torch.int32)


def _tagged(vals_f16: np.ndarray, call: int) -> np.ndarray:
    return (vals_f16.view(np.uint16).astype(np.uint32) | np.uint32((call & 0xFFFF) << 16)).view(np.int32)


def test_region_bytes():
    L = abi().lib()
    for rows in (16, 1024, 3584, 11008):
        assert L.dq_gather_region_bytes(rows) == _layout(rows)[2]
    assert L.dq_gather_region_bytes(0) == 0 and L.dq_gather_region_bytes(100) == 0


def _own_rows(wts, x):
    """This rank's rows as the gathering kernel computes them: a world-1 call
    on a region of its own."""
    region = torch.zeros(_layout(wts.d_out)[2], dtype=torch.uint8, device="cuda")
    y = torch.empty(wts.d_out, dtype=torch.float16, device="cuda")
    assert _gather(wts, x, y, _desc(0, 1, wts.d_out, wts.d_out, [region])) == 0
    return y


def test_world_one_is_the_split_gemv():
    import oracle as O
    from dyn_quant import synth
    rows_per, d_in = 1024, 4096
    w = synth.weights(rows_per, d_in, seed=3)
    packed, scales, zeros = O.quantize(w)
    wts = _weights(rows_per, d_in, seed=3)
    region = torch.zeros(_layout(rows_per)[2], dtype=torch.uint8, device="cuda")
    g = _desc(0, 1, rows_per, rows_per, [region])
    for call in range(1, 4):
        xh = synth.activation(d_in, 0.02, seed=30 + call)
        x = dev(xh)
        y = torch.empty(rows_per, dtype=torch.float16, device="cuda")
        assert _gather(wts, x, y, g) == 0
        torch.cuda.synchronize()
        first = host(y).copy()
        assert list(_hdr(region)) == [2 * call - 1]
        assert _gather(wts, x, y, g) == 0
        ref = abi_split_gemv(wts, x, 3.0)
        torch.cuda.synchronize()
        assert np.array_equal(host(y).view(np.int16), first.view(np.int16)), f"call {call}: not reproducible"
        check_y(first, host(ref), what=f"call {call} vs dq_split_gemv")
        y16, _, _ = O.split_gemv(packed, scales, zeros, w, xh, 3.0)
        check_y(first, y16, what=f"call {call} vs the oracle")
        assert list(_hdr(region)) == [2 * call]


@pytest.mark.parametrize("rows_per,d_in,tail", [(1024, 4096, 5), (3584, 8192, 0), (512, 11008, 16),
                                              (1024, 28672, 3)])
def test_rank0_of_two_with_planted_peer(rows_per, d_in, tail):
    from dyn_quant import synth
    d_total = 2 * rows_per - tail
    wts = _weights(rows_per, d_in, seed=4)
    total = _layout(rows_per)[2]
    r0 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    r1 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    g = _desc(0, 2, rows_per, d_total, [r0, r1])
    rng = np.random.default_rng(5)
    for call in range(1, 4):
        par = call & 1
        x = dev(synth.activation(d_in, 0.02, seed=40 + call))
        # rank 1 has stored its rows of this call in rank 0's copy, tagged
        peer_rows = rng.standard_normal(d_total - rows_per).astype(np.float16)
        _words(r0, rows_per, par, d_total)[rows_per:].copy_(dev(_tagged(peer_rows, call)))
        y = torch.full((d_total,), float("nan"), dtype=torch.float16, device="cuda")
        assert _gather(wts, x, y, g) == 0
        own = _own_rows(wts, x)
        torch.cuda.synchronize()
        yh = host(y)
        assert np.array_equal(yh[:rows_per].view(np.int16), host(own).view(np.int16)), f"call {call}: own rows"
        assert np.array_equal(yh[rows_per:].view(np.int16), peer_rows.view(np.int16)), f"call {call}: peer rows"
        # rank 0 stored its rows, tagged with this call, in rank 1's copy of this parity
        theirs = host(_words(r1, rows_per, par, rows_per))
        assert np.array_equal(theirs, _tagged(host(own), call)), f"call {call}: rows sent"
        assert list(_hdr(r0)) == [call], f"call {call}: calls completed"
    err = C.c_uint32(0)
    assert abi().lib().dq_read_device_error(C.byref(err), 0) == 0 and err.value & 16 == 0


def test_wait_runs_out():
    """Nothing from the other rank: the bounded waits give up (about a second)."""
    from dyn_quant import synth
    _lib = abi()
    rows_per, d_in = 256, 4096
    total = _layout(rows_per)[2]
    wts = _weights(rows_per, d_in, seed=6)
    r0 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    r1 = torch.zeros(total, dtype=torch.uint8, device="cuda")
    g = _desc(0, 2, rows_per, 2 * rows_per, [r0, r1])
    x = dev(synth.activation(d_in, 0.02, seed=7))
    y = torch.full((2 * rows_per,), 7.0, dtype=torch.float16, device="cuda")
    err = C.c_uint32(0)
    assert _lib.lib().dq_read_device_error(C.byref(err), 1) == 0
    assert _gather(wts, x, y, g) == 0
    torch.cuda.synchronize()
    assert _lib.lib().dq_read_device_error(C.byref(err), 1) == 0
    own = _own_rows(wts, x)
    torch.cuda.synchronize()
    assert err.value & 16, f"error word {err.value:#x}: the wait should have run out"
    yh = host(y)
    assert np.array_equal(yh[:rows_per].view(np.int16), host(own).view(np.int16))
    assert (yh[rows_per:] == 7.0).all()


def test_bad_arguments():
    _lib = abi()
    L = _lib.lib()
    rows_per, d_in = 256, 4096
    wts = _weights(rows_per, d_in, seed=8)
    region = torch.zeros(_layout(rows_per)[2], dtype=torch.uint8, device="cuda")
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
    small = torch.zeros(256 + 16 * 8 * 1024, dtype=torch.uint8, device="cuda")
    assert L.dq_split_gemv_gather(C.byref(wts), _ptr(x), _ptr(y), 3.0, _ptr(small), small.numel(),
                                  C.byref(_desc(0, 1, rows_per, rows_per, [region])), stream_ptr()) == \
        _lib.DQ_ERR_WORKSPACE
    torch.cuda.synchronize()
