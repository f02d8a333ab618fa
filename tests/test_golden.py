"""The oracle against the golden fixtures made from the reference's own code
(tests/golden/make_golden.py): the reference's host quantizer (bit-exact) and
the reference's GPU kernels on the B200 (GEMV outputs, detector)."""
import glob
import os

import numpy as np
import pytest

import oracle as O
from dq_testutil import MASK_BAND, check_y

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
QUANT = sorted(glob.glob(os.path.join(GOLDEN, "quant_*.npz")))
GEMV = sorted(glob.glob(os.path.join(GOLDEN, "gemv_*.npz")))


def f16(a):
    return np.asarray(a).view(np.float16)


def test_fixtures_present():
    assert len(QUANT) >= 4
    assert len(GEMV) >= 3


@pytest.mark.parametrize("path", QUANT, ids=[os.path.basename(p) for p in QUANT])
def test_oracle_quantizer_matches_reference_fixture(path):
    g = np.load(path)
    p, s, z = O.quantize(f16(g["w"]))
    assert np.array_equal(p, g["packed"])
    assert np.array_equal(s.view(np.uint16), g["scales"])
    assert np.array_equal(z.view(np.uint16), g["zeros"])


@pytest.mark.parametrize("path", GEMV, ids=[os.path.basename(p) for p in GEMV])
def test_oracle_gemvs_match_reference_kernels(path):
    g = np.load(path)
    w, x, k = f16(g["w"]), f16(g["x"]), float(g["k"])
    p, s, z = O.quantize(w)
    y16, y32, mask = O.split_gemv(p, s, z, w, x, k)
    rows = np.nonzero(g["split_rows"])[0]
    check_y(f16(g["y_split"]), y16, what="reference split kernel", rows=rows)
    y4, _ = O.int4_gemv(p, s, z, x)
    check_y(f16(g["y_int4"]), y4, what="reference INT4 kernel")
    yr, _ = O.reference_gemv(w, x)
    check_y(f16(g["y_ref"]), yr, what="reference FP16 kernel")
    # detector: the reference's index list (its own order) as a set, statistics to FP32 rounding
    mask_o, idx_o, stats_o = O.detect(x, k)
    ref_set = set(int(i) for i in g["indices"])
    ours = set(int(i) for i in np.nonzero(mask_o)[0])
    diff = ref_set ^ ours
    if diff:
        xf = x.astype(np.float64)
        margin = np.abs(np.abs(xf[sorted(diff)] - stats_o[0]) - stats_o[1])
        assert (margin <= MASK_BAND * abs(stats_o[1])).all(), sorted(diff)[:8]
    np.testing.assert_allclose(stats_o[:2], g["stats"][:2], rtol=1e-5, atol=1e-6)
