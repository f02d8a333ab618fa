"""CPU checks of the oracle itself: its FP16 conversions, its quantizer against
the reference's own quantizer (oracle/_ref/ref_quant, built from the unmodified
reference header), its detector against the reference's definition, and its
GEMVs against each other and a binary64 dense product."""
import numpy as np
import pytest

import oracle as O
from dyn_quant import synth
from dq_testutil import rel_l2


def test_f16_conversions_match_ieee():
    rng = np.random.default_rng(0)
    f = (rng.standard_normal(200000).astype(np.float32) *
         np.float32(10.0) ** rng.integers(-9, 6, 200000).astype(np.float32))
    f = np.concatenate([f, np.array([65504, 65519.99, 65520, 1e-8, 2.98e-8, 2.99e-8, 5.96e-8, -0.0,
                                     0.0, np.inf, -np.inf, 6.1e-5, 6.09e-5], np.float32)])
    with np.errstate(over="ignore"):
        expect = f.astype(np.float16)
    assert np.array_equal(O.f2h_bits(f).view(np.uint16), expect.view(np.uint16))
    h = np.arange(65536, dtype=np.uint16).view(np.float16)
    hf = O.h2f(h)
    ok = (hf.view(np.uint32) == h.astype(np.float32).view(np.uint32)) | np.isnan(hf)
    assert ok.all()


@pytest.mark.skipif(not O.ref_quant_available(), reason="reference quantizer not built")
@pytest.mark.parametrize("d_out,d_in,seed", [(64, 256, 0), (300, 1024, 1), (33, 4096, 2), (8, 11008, 3)])
def test_quantizer_bit_exact_with_reference_binary(d_out, d_in, seed):
    w = synth.weights(d_out, d_in, seed=seed)
    for a, b in zip(O.quantize(w), O.ref_quantize(w)):
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.skipif(not O.ref_quant_available(), reason="reference quantizer not built")
def test_quantizer_edge_values_bit_exact_with_reference_binary():
    w = np.zeros((10, 256), np.float16)
    w[1, :] = 1.5                     # constant group: range < 1e-8 -> scale 1
    w[2, ::2] = -0.0                  # signed zeros: first-seen tie rule
    w[3, 5] = np.inf
    w[4, 7] = -np.inf
    w[5, 9] = np.nan
    w[6, :128] = np.nan               # all-NaN group
    w[7, 3], w[7, 4] = 65504, -65504  # extreme range
    w[8, 130:140] = np.float16(6e-8)  # subnormals
    w[9, :] = np.linspace(-1, 1, 256).astype(np.float16)
    for a, b in zip(O.quantize(w), O.ref_quantize(w)):
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_quantizer_roundtrip_error_bound():
    w = synth.weights(128, 1024, seed=5)
    packed, scales, zeros = O.quantize(w)
    lo = (packed & 0xF).astype(np.float32)
    hi = (packed >> 4).astype(np.float32)
    q = np.empty((128, 1024), np.float32)
    q[:, 0::2], q[:, 1::2] = lo, hi
    s = np.repeat(scales.astype(np.float32), 128, axis=1)
    z = np.repeat(zeros.astype(np.float32), 128, axis=1)
    deq = s * (q - z)
    # half a quantization step plus FP16 rounding of scale and zero
    assert np.all(np.abs(deq - w.astype(np.float32)) <= 0.5 * s + 0.02 * s * 15 + 1e-6)


def _detect_reference_definition(x, k):
    """The detector's set from its definition in binary64 (mean, unbiased var)."""
    xf = x.astype(np.float64)
    mean = xf.mean()
    var = xf.var(ddof=1)
    thresh = k * np.sqrt(max(var, 1e-8))
    return np.abs(xf - mean) > thresh, mean, thresh


@pytest.mark.parametrize("d_in,frac,k,dist", [(4096, 0.02, 3.0, "normal"), (11008, 0.01, 3.0, "normal"),
                                              (8192, 0.05, 2.0, "t3"), (28672, 0.03, 3.0, "normal")])
def test_detector_matches_definition(d_in, frac, k, dist):
    x = synth.activation(d_in, frac, seed=1, dist=dist)
    mask, idx, stats = O.detect(x, k)
    ref, mean, thresh = _detect_reference_definition(x, k)
    assert abs(stats[0] - mean) <= 1e-5 * (1 + abs(mean))
    assert abs(stats[1] - thresh) <= 1e-5 * thresh
    diff = np.nonzero(mask.astype(bool) != ref)[0]
    near = np.abs(np.abs(x.astype(np.float64)[diff] - mean) - thresh) <= 1e-5 * thresh
    assert near.all()
    # list order: stripe class (c//32)%4 major, ascending inside
    cls = (idx // 32) % 4
    assert np.all(np.diff(cls) >= 0)
    for c in range(4):
        assert np.all(np.diff(idx[cls == c]) > 0)


def test_detector_capacity_per_stripe():
    d_in = 1024
    x = synth.activation(d_in, 0.0, seed=3)
    mask, idx, _ = O.detect(x, 0.01)
    cap = (d_in // 4) // 4
    cls = (np.arange(d_in) // 32) % 4
    for c in range(4):
        sel = np.nonzero(mask.astype(bool) & (cls == c))[0]
        assert len(sel) == cap
        # the kept ones are the first cap outliers of that class in ascending order
        flagged = np.nonzero((np.abs(x.astype(np.float32) - x.astype(np.float32).mean()) > 0) & (cls == c))[0]
        assert sel[-1] <= flagged[-1]


def test_split_equals_int4_without_outliers():
    w = synth.weights(64, 1024, seed=0)
    x = synth.activation(1024, 0.0, seed=2)
    packed, scales, zeros = O.quantize(w)
    y16s, y32s = O.split_gemv_masked(packed, scales, zeros, w, x, np.zeros(1024, np.uint8))
    y16i, y32i = O.int4_gemv(packed, scales, zeros, x)
    # same products, different pairing of the additions
    np.testing.assert_allclose(y32s, y32i, rtol=1e-5, atol=1e-5)


def test_split_beats_int4_with_outliers():
    w = synth.weights(512, 4096, seed=0)
    x = synth.activation(4096, 0.02, seed=1)
    packed, scales, zeros = O.quantize(w)
    y16s, _, mask = O.split_gemv(packed, scales, zeros, w, x, 3.0)
    y16i, _ = O.int4_gemv(packed, scales, zeros, x)
    yd = O.dense_gemv_f64(w, x)
    assert mask.sum() > 0
    assert rel_l2(y16s, yd) < 0.5 * rel_l2(y16i, yd)
    y16r, _ = O.reference_gemv(w, x)
    assert rel_l2(y16r, yd) < 1e-3


def test_split_all_outliers_is_fp16_gemv():
    w = synth.weights(32, 512, seed=4)
    x = synth.activation(512, 0.0, seed=5)
    packed, scales, zeros = O.quantize(w)
    y16s, y32s = O.split_gemv_masked(packed, scales, zeros, w, x, np.ones(512, np.uint8))
    yd = O.dense_gemv_f64(w, x)
    np.testing.assert_allclose(y32s, yd, rtol=1e-5, atol=1e-5)


def test_synthetic_outlier_counts():
    # round(frac * d_in) injected channels, as the benchmark configurations state
    for d_in, frac, n in [(4096, 0.02, 82), (4096, 0.01, 41), (11008, 0.01, 110), (8192, 0.03, 246),
                          (28672, 0.03, 860), (14336, 0.02, 287)]:
        base = synth.activation(d_in, 0.0, seed=1).astype(np.float32)
        x = synth.activation(d_in, frac, seed=1).astype(np.float32)
        assert np.count_nonzero(x != base) in range(n - 2, n + 1)  # a product can round back
