"""Host-side behaviour of the Python API that needs no GPU."""
import pytest
import torch

import dyn_quant
from dyn_quant import DynQuantLinear


def test_extension_loads_and_exports_reference_names():
    assert dyn_quant._EXTENSION_LOADED
    for name in ("quantize_weights", "split_gemv", "int4_gemv", "reference_gemv"):
        assert hasattr(dyn_quant._C, name)
    for name in ("DynQuantLinear", "quantize", "split_gemv", "int4_gemv", "reference_gemv"):
        assert hasattr(dyn_quant, name)


def test_module_construction_matches_reference():
    lin = DynQuantLinear(4096, 11008, outlier_k=2.5)
    assert (lin.d_in, lin.d_out, lin.outlier_k) == (4096, 11008, 2.5)
    assert lin.packed is None and lin.fp16_w is None
    assert "d_in=4096" in repr(lin)
    with pytest.raises(RuntimeError, match="load_weight"):
        lin(torch.zeros(4096, dtype=torch.float16))


def test_load_weight_checks_shape():
    lin = DynQuantLinear(256, 16)
    with pytest.raises(AssertionError):
        lin.load_weight(torch.zeros(16, 128, dtype=torch.float16))


def test_cpu_tensors_are_rejected_not_computed_on_cpu():
    # no CPU fallback: the binding refuses host tensors
    w = torch.zeros(16, 256, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        dyn_quant.quantize(w)
    p = torch.zeros(16, 128, dtype=torch.uint8)
    s = torch.zeros(16, 2, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        dyn_quant.split_gemv(p, s, s, w, torch.zeros(256, dtype=torch.float16))
    with pytest.raises(RuntimeError):
        dyn_quant.reference_gemv(w, torch.zeros(256, dtype=torch.float16))
