"""The reference's C++ host API restated over the C ABI
(include/dq_reference_api.hpp): quantize_weights_host, launch_split_gemv,
launch_int4_gemv, launch_reference_gemv and free_quantized_weights give the
oracle's results when called exactly as code written for the reference calls
them."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import _lib, synth  # noqa: E402
from dq_testutil import check_y, dev, host  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("refapi") / "librefapi.so")
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(cuda, "include"), os.path.join(ROOT, "tests", "cpp", "ref_api_harness.cpp"),
           "-o", out, "-L", lib_dir, "-ldq_b200", "-L", os.path.join(cuda, "lib64"), "-lcudart",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True)
    h = C.CDLL(out)
    h.refapi_run.restype = C.c_int
    h.refapi_run.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p,
                             C.c_void_p, C.c_void_p, C.c_int]
    return h


@pytest.mark.parametrize("d_out,d_in,frac", [(4096, 4096, 0.02), (1024, 11008, 0.01), (100, 256, 0.05)])
def test_reference_signatures_match_oracle(harness, d_out, d_in, frac):
    torch.cuda.set_device(0)
    w = synth.weights(d_out, d_in, seed=0)
    x = synth.activation(d_in, frac, seed=1)
    x_t = dev(x)
    y_split = torch.empty(d_out, dtype=torch.float16, device="cuda")
    y_int4 = torch.empty_like(y_split)
    y_ref = torch.empty_like(y_split)
    packed = np.empty((d_out, d_in // 2), np.uint8)
    st = harness.refapi_run(w.ctypes.data, d_out, d_in, x_t.data_ptr(), 3.0, y_split.data_ptr(), y_int4.data_ptr(),
                            y_ref.data_ptr(), packed.ctypes.data, 2)
    assert st == 0, st
    p_o, s_o, z_o = O.quantize(w)
    assert np.array_equal(packed, p_o)
    y16, y32, _ = O.split_gemv(p_o, s_o, z_o, w, x, 3.0)
    check_y(host(y_split), y16, y32, what="launch_split_gemv")
    y4, _ = O.int4_gemv(p_o, s_o, z_o, x)
    check_y(host(y_int4), y4, what="launch_int4_gemv")
    yr, _ = O.reference_gemv(w, x)
    check_y(host(y_ref), yr, what="launch_reference_gemv")
