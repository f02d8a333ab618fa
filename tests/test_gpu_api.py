"""The Python API (dyn_quant.*, DynQuantLinear) on the GPU, mirroring the
reference's tests/test_python.py (its three tests, with the FP32 reference
computed in one dtype -- the reference's own version mixes fp16 and fp32 in
torch.matmul and raises before asserting) plus parity against the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import dyn_quant  # noqa: E402
from dyn_quant import DynQuantLinear, quantize, split_gemv  # noqa: E402
import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dq_testutil import check_y, host  # noqa: E402

D_IN = 4096
D_OUT = 4096
OUTLIER_FRAC = 0.05
OUTLIER_MAG = 20.0
OUTLIER_K = 3.0
COSINE_THRESHOLD = 0.9999


def generate_outlier_activation(d_in, frac, mag):
    x = torch.randn(d_in, dtype=torch.float16, device="cuda")
    n_out = int(frac * d_in)
    x[:n_out] = (torch.randn(n_out, device="cuda") * mag).half()
    return x


def cosine_sim(a, b):
    return float(torch.nn.functional.cosine_similarity(a.float().unsqueeze(0), b.float().unsqueeze(0)).item())


def fp32_ref(weight, x):
    return (weight.float() @ x.float()).half()


def oracle_outputs(weight, x, k=OUTLIER_K):
    """The oracle's split and INT4 outputs on the same inputs (host copies)."""
    w = weight.cpu().numpy()
    xh = x.cpu().numpy()
    packed, scales, zeros = O.quantize(w)
    y16, y32, _ = O.split_gemv(packed, scales, zeros, w, xh, k)
    y4, _ = O.int4_gemv(packed, scales, zeros, xh)
    return y16, y32, y4


def cos_np(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


# The reference's own gate, cosine(split, FP16 GEMV) >= 0.9999
# (tests/test_python.py:15,48 and tests/test_correctness.cu:113), is not met by
# its algorithm on its own input distribution: INT4 group-128 quantisation of
# N(0, 0.02) weights alone gives about 0.995, and the oracle's split result
# reaches about 0.9994-0.9995 here.  The tests below keep the reference's data
# generation and assert what the algorithm does deliver: the same output as the
# oracle on the same inputs, and split strictly better than INT4-only.


def test_dyn_quant_linear():
    torch.manual_seed(0)
    weight = torch.randn(D_OUT, D_IN, dtype=torch.float16, device="cuda") * 0.02
    x = generate_outlier_activation(D_IN, OUTLIER_FRAC, OUTLIER_MAG)
    linear = DynQuantLinear(D_IN, D_OUT, outlier_k=OUTLIER_K)
    linear.load_weight(weight)
    linear.cuda()
    y = linear(x)
    assert y.shape == (D_OUT,) and y.dtype == torch.float16
    y16, y32, y4 = oracle_outputs(weight, x)
    check_y(host(y), y16, what="DynQuantLinear vs oracle")
    ref = host(fp32_ref(weight, x))
    assert abs(cos_np(host(y), ref) - cos_np(y16, ref)) < 1e-5
    assert cos_np(host(y), ref) > cos_np(y4, ref)


def test_functional_api():
    torch.manual_seed(1)
    weight = torch.randn(D_OUT, D_IN, dtype=torch.float16, device="cuda") * 0.02
    x = generate_outlier_activation(D_IN, OUTLIER_FRAC, OUTLIER_MAG)
    packed, scales, zeros, fp16_copy = quantize(weight)
    assert packed.shape == (D_OUT, D_IN // 2) and packed.dtype == torch.uint8
    assert scales.shape == (D_OUT, D_IN // 128) and zeros.dtype == torch.float16
    assert torch.equal(fp16_copy, weight)
    y = split_gemv(packed, scales, zeros, fp16_copy, x, OUTLIER_K)
    y16, y32, y4 = oracle_outputs(weight, x)
    check_y(host(y), y16, what="split_gemv vs oracle")


def test_int4_vs_split_with_outliers():
    torch.manual_seed(2)
    weight = torch.randn(D_OUT, D_IN, dtype=torch.float16, device="cuda") * 0.02
    x = generate_outlier_activation(D_IN, OUTLIER_FRAC, OUTLIER_MAG)
    packed, scales, zeros, fp16_copy = quantize(weight)
    y_ref = host(fp32_ref(weight, x))
    y_int4 = host(dyn_quant.int4_gemv(packed, scales, zeros, fp16_copy, x))
    y_split = host(dyn_quant.split_gemv(packed, scales, zeros, fp16_copy, x, OUTLIER_K))
    y16, _, y4 = oracle_outputs(weight, x)
    check_y(y_int4, y4, what="int4_gemv vs oracle")
    check_y(y_split, y16, what="split_gemv vs oracle")
    assert cos_np(y_split, y_ref) > cos_np(y_int4, y_ref) + 1e-3


@pytest.mark.parametrize("d_out,d_in,frac", [(4096, 4096, 0.02), (11008, 4096, 0.01), (4096, 11008, 0.01)])
def test_module_matches_oracle(d_out, d_in, frac):
    w = synth.weights(d_out, d_in, seed=0)
    x = synth.activation(d_in, frac, seed=1)
    lin = DynQuantLinear(d_in, d_out, 3.0)
    lin.load_weight(torch.from_numpy(w).cuda())
    y = host(lin(torch.from_numpy(x).cuda()))
    packed, scales, zeros = O.quantize(w)
    assert np.array_equal(host(lin.packed), packed)
    assert np.array_equal(host(lin.scales).view(np.uint16), scales.view(np.uint16))
    mask = host(dyn_quant.detect_outliers(torch.from_numpy(x).cuda(), 3.0)[0])
    y16, y32 = O.split_gemv_masked(packed, scales, zeros, w, x, mask.astype(np.uint8))
    check_y(y, y16, y32, what="DynQuantLinear")
    y16o, _, _ = O.split_gemv(packed, scales, zeros, w, x, 3.0)
    check_y(y, y16o, what="DynQuantLinear vs oracle detection")


def test_fp16_w_is_a_view_of_the_mirror():
    w = synth.weights(256, 512, seed=4)
    lin = DynQuantLinear(512, 256)
    lin.load_weight(torch.from_numpy(w).cuda())
    assert lin.fp16_w.shape == (256, 512)
    assert not lin.fp16_w.is_contiguous() and lin.fp16_w.t().is_contiguous()
    assert np.array_equal(host(lin.fp16_w).view(np.uint16), w.view(np.uint16))
    # the functional API takes either layout and gives the same bits
    x = torch.from_numpy(synth.activation(512, 0.03, seed=5)).cuda()
    a = split_gemv(lin.packed, lin.scales, lin.zeros, lin.fp16_w, x, 3.0)
    b = split_gemv(lin.packed, lin.scales, lin.zeros, lin.fp16_w.contiguous(), x, 3.0)
    assert torch.equal(a, b)


def test_state_dict_round_trip():
    w = torch.from_numpy(synth.weights(512, 1024, seed=6)).cuda()
    x = torch.from_numpy(synth.activation(1024, 0.02, seed=7)).cuda()
    a = DynQuantLinear(1024, 512, 2.5)
    a.load_weight(w)
    sd = a.state_dict()
    b = DynQuantLinear(1024, 512, 2.5)
    b.load_state_dict(sd)
    assert torch.equal(a(x), b(x))
    c = DynQuantLinear(1024, 512, 2.5)
    c.load_state_dict({k: v.cpu() for k, v in sd.items()})
    assert torch.equal(a(x), c(x))


def test_errors_raise_runtime_error():
    lin = DynQuantLinear(256, 16)
    with pytest.raises(RuntimeError):
        lin(torch.zeros(256, dtype=torch.float16, device="cuda"))
    w = torch.zeros(16, 256, dtype=torch.float16, device="cuda")
    p, s, z, f = quantize(w)
    with pytest.raises(RuntimeError):
        split_gemv(p, s, z, f, torch.zeros(128, dtype=torch.float16, device="cuda"))
    with pytest.raises(RuntimeError):
        split_gemv(p, s, z, f, torch.zeros(256, dtype=torch.float32, device="cuda"))
    with pytest.raises(RuntimeError):
        split_gemv(p.cpu(), s, z, f, torch.zeros(256, dtype=torch.float16, device="cuda"))
    with pytest.raises(RuntimeError):
        quantize(torch.zeros(16, 100, dtype=torch.float16, device="cuda"))


def test_misaligned_activation_view_is_rehomed():
    w = synth.weights(64, 256, seed=8)
    p, s, z, f = quantize(torch.from_numpy(w).cuda())
    buf = torch.from_numpy(synth.activation(257, 0.0, seed=9)).cuda()
    x = buf[1:]  # 2-byte offset view
    assert x.data_ptr() % 16 != 0
    y1 = split_gemv(p, s, z, f, x, 3.0)
    y2 = split_gemv(p, s, z, f, x.clone(), 3.0)
    assert torch.equal(y1, y2)


def test_forward_handle_follows_the_module():
    """forward() on one vector goes through the prebuilt weights handle once
    the module holds it; the result is the functional call's, bit for bit,
    and the handle is rebuilt when the weights, k or the device placement of
    the buffers change."""
    d_out, d_in = 1024, 2048
    w = torch.from_numpy(synth.weights(d_out, d_in, seed=11)).cuda()
    x = torch.from_numpy(synth.activation(d_in, 0.02, seed=12)).cuda()
    lin = DynQuantLinear(d_in, d_out, 3.0)
    lin.load_weight(w)

    def functional(m, v):
        return split_gemv(m.packed, m.scales, m.zeros, m.fp16_w, v, m.outlier_k, m._native)

    y0 = lin(x)  # first call: general path, builds the handle
    assert lin.__dict__.get("_fast") is not None
    assert torch.equal(lin(x), y0) and torch.equal(y0, functional(lin, x))
    assert torch.equal(lin(x.view(1, d_in)), y0)
    assert torch.equal(lin(x.float()), y0)  # not float16: general path, same result
    xs = torch.from_numpy(synth.activation(d_in + 128, 0.02, seed=13)).cuda()[1:1 + d_in]
    assert xs.data_ptr() % 16 != 0
    assert torch.equal(lin(xs), functional(lin, xs.clone()))
    # out=: y written into a slice of a larger buffer, the slice returned
    buf = torch.zeros(d_out + 64, dtype=torch.float16, device="cuda")
    o = buf[8:8 + d_out]
    r = lin(x, out=o)
    assert r.data_ptr() == o.data_ptr() and torch.equal(o, y0)
    assert torch.equal(buf[:8], torch.zeros(8, dtype=torch.float16, device="cuda"))
    assert torch.equal(lin(x.float(), out=o), y0)  # general path, same result
    with pytest.raises(RuntimeError):
        lin(x, out=buf[:d_out - 1])
    # batches still take the batched path
    xb = torch.stack([x, x.flip(0)])
    assert lin(xb).shape == (2, d_out)
    # new k: the handle must not keep the old threshold
    lin.outlier_k = 1.5
    y_k = lin(x)
    assert torch.equal(y_k, functional(lin, x))
    assert not torch.equal(y_k, y0)
    # new weights: a rebuilt handle
    lin.load_weight(-w)
    y_neg = lin(x)
    assert torch.equal(y_neg, functional(lin, x))
    assert not torch.equal(y_neg, y_k)
    # a module moved off the GPU and back keeps working
    lin.cpu()
    assert lin.__dict__.get("_fast") is None
    lin.cuda()
    assert torch.equal(lin(x), y_neg)
    # the handle does not travel with a copy of the module
    import copy
    dup = copy.deepcopy(lin)
    assert torch.equal(dup(x), y_neg)
