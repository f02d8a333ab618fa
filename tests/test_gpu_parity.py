"""GPU parity of the C ABI (libdq_b200.so) against the oracle.

Every call goes through include/dq_abi.h via ctypes; inputs are seeded
synthetic tensors with the benchmark shapes and value distributions.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dq_testutil import (  # noqa: E402
    abi, abi_build_native, abi_colmajor, abi_detect, abi_int4_gemv, abi_quantize, abi_reference_gemv, abi_split_gemv,
    abi_weights, check_mask, check_y, dev, host,
)

# (d_out, d_in, outlier fraction, k, activation distribution)
CASES = [
    (4096, 4096, 0.02, 3.0, "normal"),    # Llama-2-7B q_proj, 2 % outliers
    (1024, 11008, 0.01, 3.0, "normal"),   # 7B down-proj input width
    (2048, 8192, 0.03, 3.0, "normal"),    # 70B q_proj input width
    (512, 28672, 0.03, 3.0, "normal"),    # 70B down-proj input width (four column slabs)
    (1000, 16384, 0.03, 3.0, "normal"),   # long rows without slabs, ragged last row block
    (100, 256, 0.05, 3.0, "normal"),      # ragged d_out
    (17, 128, 0.05, 2.0, "normal"),       # smallest d_in
    (1, 4096, 0.02, 3.0, "normal"),       # one row
    (4096, 4096, 0.0, 3.0, "normal"),     # no injected outliers
    (1024, 4096, 0.10, 2.0, "normal"),    # many outliers
    (1024, 8192, 0.05, 3.0, "t3"),        # heavy-tailed activations
    (1024, 8192, 0.0, 6.0, "normal"),     # nothing above 6 sigma
]
IDS = [f"{a}x{b}-f{c}-k{d}-{e}" for a, b, c, d, e in CASES]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)


_cache = {}


def make_case(d_out, d_in, frac, dist, seed_x=1):
    key = (d_out, d_in, frac, dist, seed_x)
    if key not in _cache:
        w = synth.weights(d_out, d_in, seed=0)
        x = synth.activation(d_in, frac, seed=seed_x, dist=dist)
        packed, scales, zeros = O.quantize(w)
        _cache.clear()
        _cache[key] = (w, x, packed, scales, zeros)
    return _cache[key]


@pytest.mark.parametrize("d_out,d_in,frac,k,dist", CASES, ids=IDS)
def test_quantize_bit_exact(d_out, d_in, frac, k, dist):
    w, x, packed, scales, zeros = make_case(d_out, d_in, frac, dist)
    p, s, z = abi_quantize(dev(w))
    torch.cuda.synchronize()
    assert np.array_equal(host(p), packed)
    assert np.array_equal(host(s).view(np.uint16), scales.view(np.uint16))
    assert np.array_equal(host(z).view(np.uint16), zeros.view(np.uint16))


def test_quantize_edge_values_bit_exact():
    w = np.zeros((8, 256), np.float16)
    w[1, :] = 1.5
    w[2, ::2] = -0.0
    w[3, 5] = np.inf
    w[4, 7] = -np.inf
    w[5, 9] = np.nan
    w[6, :128] = np.nan
    w[7, 3] = 65504
    w[7, 4] = -65504
    w[0, 130:140] = np.float16(6e-8)
    ref = O.quantize(w)
    got = abi_quantize(dev(w))
    for r, g in zip(ref, got):
        assert np.array_equal(host(g).view(np.uint8), r.view(np.uint8))


def test_colmajor_mirror():
    w = synth.weights(300, 384, seed=3)
    cm = abi_colmajor(dev(w))
    assert np.array_equal(host(cm).view(np.uint16), np.ascontiguousarray(w.T).view(np.uint16))


@pytest.mark.parametrize("d_out,d_in,frac,k,dist", CASES, ids=IDS)
def test_detect_matches_oracle(d_out, d_in, frac, k, dist):
    _, x, *_ = make_case(d_out, d_in, frac, dist)
    mask, idx, stats = abi_detect(dev(x), k)
    rmask, ridx, rstats = O.detect(x, k)
    # mean / threshold agree to FP32 rounding of differently ordered sums
    assert abs(stats[0] - rstats[0]) <= 1e-5 * (1 + abs(rstats[0]))
    assert abs(stats[1] - rstats[1]) <= 1e-5 * abs(rstats[1])
    ndiff = check_mask(mask, rmask, x.astype(np.float32), float(rstats[0]), float(rstats[1]))
    assert mask.sum() == len(idx) <= d_in // 4
    if ndiff == 0:
        # same set and the reference's list order (stripe class 0 ascending, then 1, 2, 3)
        assert np.array_equal(idx, ridx)


@pytest.mark.parametrize("layout", ["colmajor+native", "colmajor", "rowmajor+native", "rowmajor"])
@pytest.mark.parametrize("d_out,d_in,frac,k,dist", CASES, ids=IDS)
def test_split_gemv_matches_oracle(d_out, d_in, frac, k, dist, layout):
    w, x, packed, scales, zeros = make_case(d_out, d_in, frac, dist)
    w_t, x_t = dev(w), dev(x)
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    nat = abi_build_native(p_t, s_t, z_t) if layout.endswith("native") else None
    if layout.startswith("colmajor"):
        wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(w_t), native=nat)
    else:
        wts = abi_weights(p_t, s_t, z_t, w_rm=w_t, native=nat)
    y = host(abi_split_gemv(wts, x_t, k))
    gmask, _, _ = abi_detect(x_t, k)
    # the GEMV arithmetic, given the mask the GPU applies
    y16m, y32m = O.split_gemv_masked(packed, scales, zeros, w, x, gmask.astype(np.uint8))
    check_y(y, y16m, y32m, what="split(gpu mask)")
    # end to end against the oracle's own detection
    y16, y32, _ = O.split_gemv(packed, scales, zeros, w, x, k)
    check_y(y, y16, None, what="split(oracle mask)")


@pytest.mark.parametrize("native", [True, False])
@pytest.mark.parametrize("d_out,d_in,frac,k,dist", CASES[:8], ids=IDS[:8])
def test_int4_gemv_matches_oracle(d_out, d_in, frac, k, dist, native):
    w, x, packed, scales, zeros = make_case(d_out, d_in, frac, dist)
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    wts = abi_weights(p_t, s_t, z_t, native=abi_build_native(p_t, s_t, z_t) if native else None)
    x_t = dev(x)
    y = host(abi_int4_gemv(wts, x_t))
    y16, y32 = O.int4_gemv(packed, scales, zeros, x)
    check_y(y, y16, y32, what="int4")


@pytest.mark.parametrize("d_out,d_in,frac,k,dist", CASES[:8], ids=IDS[:8])
def test_reference_gemv_matches_oracle(d_out, d_in, frac, k, dist):
    w, x, *_ = make_case(d_out, d_in, frac, dist)
    y = host(abi_reference_gemv(dev(w), dev(x)))
    y16, y32 = O.reference_gemv(w, x)
    check_y(y, y16, y32, what="fp16 gemv")


@pytest.mark.parametrize("d_in", [2048, 16384, 28672])
def test_capacity_rule_many_outliers(d_in):
    # k = 0.05 flags most channels; the per-stripe capacity (d_in/16) must trim
    # them (28672: rows cut into column slabs, the mask from all of x)
    x = synth.activation(d_in, 0.0, seed=11)
    mask, idx, stats = abi_detect(dev(x), 0.05)
    rmask, ridx, rstats = O.detect(x, 0.05)
    assert rmask.sum() == d_in // 4  # every stripe class saturated
    check_mask(mask, rmask, x.astype(np.float32), float(rstats[0]), float(rstats[1]))
    w = synth.weights(64, d_in, seed=2)
    packed, scales, zeros = O.quantize(w)
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(dev(w)), native=abi_build_native(p_t, s_t, z_t))
    y = host(abi_split_gemv(wts, dev(x), 0.05))
    y16m, y32m = O.split_gemv_masked(packed, scales, zeros, w, x, mask.astype(np.uint8))
    check_y(y, y16m, y32m, what="split(capacity)")


def _concentrated(d_in, first, n, mag, seed):
    """x ~ N(0, 1) with n channels of magnitude mag (random signs) among the
    first `first` columns: the outliers pile up in one or a few 512-column
    chunks."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(d_in).astype(np.float32)
    idx = rng.choice(first, n, replace=False)
    x[idx] = mag * np.sign(rng.standard_normal(n))
    return x.astype(np.float16)


@pytest.mark.parametrize("d_out,d_in,first,n", [
    (4096, 4096, 512, 20),     # one chunk, two 16-column batches
    (4096, 4096, 512, 40),     # one chunk, three 16-column batches
    (4096, 4096, 204, 150),    # the reference test's layout: the first channels
    (2048, 28672, 512, 24),    # longest rows: all outliers in the first column slab
    (1000, 8192, 1024, 70),    # ragged last row block, two chunks
])
def test_split_gemv_concentrated_outliers(d_out, d_in, first, n):
    w = synth.weights(d_out, d_in, seed=5)
    x = _concentrated(d_in, first, n, 50.0, seed=6)
    packed, scales, zeros = O.quantize(w)
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    for native in (True, False):
        wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(dev(w)),
                          native=abi_build_native(p_t, s_t, z_t) if native else None)
        y = host(abi_split_gemv(wts, dev(x), 3.0))
        y16, y32, _ = O.split_gemv(packed, scales, zeros, w, x, 3.0)
        check_y(y, y16, y32, what=f"split {d_out}x{d_in} {n} outliers in the first {first} (native={native})")


def test_constant_activation_has_no_outliers():
    x = np.full(1024, 0.75, np.float16)
    mask, idx, stats = abi_detect(dev(x), 3.0)
    assert not mask.any() and len(idx) == 0
    assert stats[2] == 0.0
    np.testing.assert_allclose(stats[1], 3.0 * 1e-4, rtol=1e-6)


def test_split_gemv_deterministic_and_stream_ordered():
    w, x, packed, scales, zeros = make_case(2048, 8192, 0.03, "normal")
    p_t, s_t, z_t = dev(packed), dev(scales), dev(zeros)
    wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(dev(w)), native=abi_build_native(p_t, s_t, z_t))
    x_t = dev(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ys = [abi_split_gemv(wts, x_t, 3.0) for _ in range(3)]
    s.synchronize()
    a = [host(v).view(np.uint16) for v in ys]
    assert np.array_equal(a[0], a[1]) and np.array_equal(a[0], a[2])


def test_native_layout():
    d_out, d_in = 37, 11008  # ragged rows, a partial last 4-group chunk (G = 86)
    rng = np.random.default_rng(5)
    packed = rng.integers(0, 256, (d_out, d_in // 2), dtype=np.uint8)
    G = d_in // 128
    s = (np.arange(d_out * G) % 7 + 1).astype(np.float16).reshape(d_out, G)
    z = (np.arange(d_out * G) % 5).astype(np.float16).reshape(d_out, G)
    got = host(abi_build_native(dev(packed), dev(s), dev(z)))
    NC = (G + 3) // 4
    n_rb = (d_out + 15) // 16
    ref = np.zeros((n_rb, NC, 4352), np.uint8)
    for rb in range(n_rb):
        for c in range(NC):
            blk = ref[rb, c]
            # piece (sl * 2 + h) * 32 + 8 t + (g ^ 2t): row rb*16 + g + 8h, group 4c + t, columns 32 sl .. +31
            for sl in range(4):
                for h in range(2):
                    for g in range(8):
                        for t in range(4):
                            row = rb * 16 + g + 8 * h
                            grp = 4 * c + t
                            if row >= d_out or grp >= G:
                                continue
                            o = ((sl * 2 + h) * 32 + 8 * t + (g ^ (2 * t))) * 16
                            blk[o:o + 16] = packed[row, 64 * grp + 16 * sl:64 * grp + 16 * sl + 16]
            sz = np.zeros((16, 4), np.uint32)
            for r in range(16):
                row = rb * 16 + r
                for jj in range(4):
                    grp = 4 * c + jj
                    if row < d_out and grp < G:
                        sz[r, jj] = int(s.view(np.uint16)[row, grp]) | (int(z.view(np.uint16)[row, grp]) << 16)
            blk[4096:] = sz.reshape(-1).view(np.uint8)
    assert np.array_equal(got, ref.reshape(-1))


def test_device_error_word_is_clear():
    import ctypes as C
    _lib = abi()
    w = C.c_uint32(99)
    assert _lib.lib().dq_read_device_error(C.byref(w), 1) == 0
    assert w.value == 0


def test_abi_rejects_bad_arguments():
    _lib = abi()
    L = _lib.lib()
    x = torch.zeros(4096 + 8, dtype=torch.float16, device="cuda")
    y = torch.empty(16, dtype=torch.float16, device="cuda")
    p = torch.zeros((16, 2048), dtype=torch.uint8, device="cuda")
    s = torch.zeros((16, 32), dtype=torch.float16, device="cuda")
    wts = abi_weights(p, s, s, w_rm=torch.zeros((16, 4096), dtype=torch.float16, device="cuda"))
    import ctypes as C
    from dq_testutil import workspace
    ws = workspace(16, 4096)
    W = (C.c_void_p(ws.data_ptr()), ws.numel())
    # misaligned x (2-byte offset)
    assert L.dq_split_gemv(C.byref(wts), C.c_void_p(x.data_ptr() + 2), C.c_void_p(y.data_ptr()), 3.0,
                           *W, None) == _lib.DQ_ERR_ALIGNMENT
    bad = abi_weights(p, s, s, w_rm=None)
    assert L.dq_split_gemv(C.byref(bad), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 3.0,
                           *W, None) == _lib.DQ_ERR_INVALID_ARGUMENT
    # workspace missing or too small
    assert L.dq_split_gemv(C.byref(wts), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 3.0,
                           None, 0, None) == _lib.DQ_ERR_WORKSPACE
    assert L.dq_split_gemv(C.byref(wts), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 3.0,
                           W[0], 64, None) == _lib.DQ_ERR_WORKSPACE
    wts.d_in = 4000
    assert L.dq_split_gemv(C.byref(wts), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 3.0,
                           *W, None) == _lib.DQ_ERR_SHAPE
    wts.d_in = 65536
    assert L.dq_split_gemv(C.byref(wts), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 3.0,
                           *W, None) == _lib.DQ_ERR_UNSUPPORTED


FULL = [("llama2_7b_gate", 11008, 4096, 0.01), ("llama2_7b_down", 4096, 11008, 0.01),
        ("llama2_70b_q", 8192, 8192, 0.03), ("llama2_70b_gate", 28672, 8192, 0.03),
        ("llama2_70b_down", 8192, 28672, 0.03)]


@pytest.mark.parametrize("name,d_out,d_in,frac", FULL, ids=[f[0] for f in FULL])
def test_split_gemv_full_size(name, d_out, d_in, frac):
    """Benchmark shapes end to end: quantize on the GPU (bit-exact), mirror,
    detect, split GEMV; checked against the oracle at full size."""
    w = synth.weights(d_out, d_in, seed=0)
    x = synth.activation(d_in, frac, seed=1)
    w_t, x_t = dev(w), dev(x)
    p_t, s_t, z_t = abi_quantize(w_t)
    packed, scales, zeros = host(p_t), host(s_t), host(z_t)
    wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(w_t), native=abi_build_native(p_t, s_t, z_t))
    del w_t
    y = host(abi_split_gemv(wts, x_t, 3.0))
    gmask, _, _ = abi_detect(x_t, 3.0)
    y16m, y32m = O.split_gemv_masked(packed, scales, zeros, w, x, gmask.astype(np.uint8))
    check_y(y, y16m, y32m, what=name)
    # accuracy against the FP16 weights in binary64: the split path must beat INT4-only
    yd = O.dense_gemv_f64(w, x)
    y4, _ = O.int4_gemv(packed, scales, zeros, x)
    from dq_testutil import rel_l2
    assert rel_l2(y, yd) < rel_l2(y4, yd)
