"""Parity against the reference's OWN kernels, run on the same B200.

oracle/_ref/libdqref_gpu.so is the reference's src/{split,int4,reference}_gemv.cu
and src/outlier_detect.cuh built for sm_100a (oracle/build_oracle.py: three
minimal compile fixes, the reference's own -use_fast_math flags).  Skipped when
that library was not built (it needs the reference sources at build time).

The reference's split_gemv_kernel stages packed bytes for rows 0..1 of every
4-row block only (src/split_gemv.cu:85-93 with a 128-thread block), so its
outputs for rows r % 4 in {2, 3} come from shared memory it never wrote; only
rows r % 4 in {0, 1} are compared for the split GEMV.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dq_testutil import (  # noqa: E402
    abi_build_native, abi_colmajor, abi_detect, abi_int4_gemv, abi_quantize, abi_reference_gemv, abi_split_gemv, abi_weights,
    check_mask, check_y, dev, host, stream_ptr,
)

if not os.path.exists(O.REF_GPU_LIB):
    pytest.skip("reference GPU build (oracle/_ref/libdqref_gpu.so) not present", allow_module_level=True)

_ref = None


def ref():
    global _ref
    if _ref is None:
        L = C.CDLL(O.REF_GPU_LIB)
        P = C.c_void_p
        L.dqref_split_gemv.argtypes = [P, P, P, P, P, P, C.c_int, C.c_int, C.c_float, P]
        L.dqref_int4_gemv.argtypes = [P, P, P, P, P, C.c_int, C.c_int, P]
        L.dqref_reference_gemv.argtypes = [P, P, P, C.c_int, C.c_int, P]
        L.dqref_detect.argtypes = [P, C.c_int, C.c_float, P, P, P, P]
        for f in (L.dqref_split_gemv, L.dqref_int4_gemv, L.dqref_reference_gemv, L.dqref_detect):
            f.restype = C.c_int
        _ref = L
    return _ref


def p(t):
    return C.c_void_p(t.data_ptr())


CASES = [(4096, 4096, 0.02), (2048, 11008, 0.01), (1024, 8192, 0.03), (256, 4096, 0.05)]


@pytest.mark.parametrize("d_out,d_in,frac", CASES)
def test_against_reference_kernels(d_out, d_in, frac):
    w = synth.weights(d_out, d_in, seed=0)
    x = synth.activation(d_in, frac, seed=1)
    w_t, x_t = dev(w), dev(x)
    p_t, s_t, z_t = abi_quantize(w_t)
    k = 3.0
    # --- reference kernels ---------------------------------------------------
    R = ref()
    y_rs = torch.empty(d_out, dtype=torch.float16, device="cuda")
    y_r4 = torch.empty_like(y_rs)
    y_rf = torch.empty_like(y_rs)
    assert R.dqref_split_gemv(p(p_t), p(s_t), p(z_t), p(w_t), p(x_t), p(y_rs), d_out, d_in, k, stream_ptr()) == 0
    assert R.dqref_int4_gemv(p(p_t), p(s_t), p(z_t), p(x_t), p(y_r4), d_out, d_in, stream_ptr()) == 0
    assert R.dqref_reference_gemv(p(w_t), p(x_t), p(y_rf), d_out, d_in, stream_ptr()) == 0
    idx = torch.empty(d_in // 4, dtype=torch.int32, device="cuda")
    cnt = torch.empty(1, dtype=torch.int32, device="cuda")
    st = torch.empty(4, dtype=torch.float32, device="cuda")
    assert R.dqref_detect(p(x_t), d_in, k, p(idx), p(cnt), p(st), stream_ptr()) == 0
    torch.cuda.synchronize()
    n = int(host(cnt)[0])
    r_idx = host(idx)[:n]
    r_stats = host(st)
    r_mask = np.zeros(d_in, bool)
    r_mask[r_idx] = True
    # --- ours ------------------------------------------------------------------
    mask, o_idx, o_stats = abi_detect(x_t, k)
    check_mask(mask, r_mask, x.astype(np.float32), float(r_stats[0]), float(r_stats[1]), "vs reference detector")
    if np.array_equal(mask, r_mask):
        assert np.array_equal(o_idx, r_idx)  # same list order
    wts = abi_weights(p_t, s_t, z_t, w_cm=abi_colmajor(w_t), native=abi_build_native(p_t, s_t, z_t))
    y = host(abi_split_gemv(wts, x_t, k))
    rows = np.nonzero(np.arange(d_out) % 4 < 2)[0]
    check_y(y, host(y_rs), rows=rows, what="split vs reference kernel (rows%4<2)")
    check_y(host(abi_int4_gemv(wts, x_t)), host(y_r4), what="int4 vs reference kernel")
    check_y(host(abi_reference_gemv(w_t, x_t)), host(y_rf), what="fp16 vs reference kernel")
    # and the oracle agrees with the reference kernels the same way
    packed, scales, zeros = host(p_t), host(s_t), host(z_t)
    y16, _, _ = O.split_gemv(packed, scales, zeros, w, x, k)
    check_y(y16, host(y_rs), rows=rows, what="oracle split vs reference kernel")
    y4, _ = O.int4_gemv(packed, scales, zeros, x)
    check_y(y4, host(y_r4), what="oracle int4 vs reference kernel")
