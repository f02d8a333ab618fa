"""The sm_100a kernels against the golden fixtures made from the reference's
own code (tests/golden/make_golden.py): quantizer bytes bit-exact against the
reference's host quantizer; GEMV outputs against the reference's GPU kernels."""
import glob
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from dq_testutil import (  # noqa: E402
    abi_build_native, abi_colmajor, abi_int4_gemv, abi_quantize, abi_reference_gemv, abi_split_gemv, abi_weights,
    check_y, dev, host,
)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
QUANT = sorted(glob.glob(os.path.join(GOLDEN, "quant_*.npz")))
GEMV = sorted(glob.glob(os.path.join(GOLDEN, "gemv_*.npz")))


def f16(a):
    return np.asarray(a).view(np.float16)


@pytest.mark.parametrize("path", QUANT, ids=[os.path.basename(p) for p in QUANT])
def test_gpu_quantizer_matches_reference_fixture(path):
    g = np.load(path)
    p, s, z = abi_quantize(dev(f16(g["w"])))
    assert np.array_equal(host(p), g["packed"])
    assert np.array_equal(host(s).view(np.uint16), g["scales"])
    assert np.array_equal(host(z).view(np.uint16), g["zeros"])


@pytest.mark.parametrize("path", GEMV, ids=[os.path.basename(p) for p in GEMV])
def test_gpu_gemvs_match_reference_kernels(path):
    g = np.load(path)
    w, x, k = f16(g["w"]), f16(g["x"]), float(g["k"])
    w_t, x_t = dev(w), dev(x)
    p_t, s_t, z_t = abi_quantize(w_t)
    wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(w_t), native=abi_build_native(p_t, s_t, z_t))
    rows = np.nonzero(g["split_rows"])[0]
    check_y(host(abi_split_gemv(wts, x_t, k)), f16(g["y_split"]), what="split vs reference kernel", rows=rows)
    check_y(host(abi_int4_gemv(wts, x_t)), f16(g["y_int4"]), what="INT4 vs reference kernel")
    check_y(host(abi_reference_gemv(w_t, x_t)), f16(g["y_ref"]), what="FP16 vs reference kernel")
