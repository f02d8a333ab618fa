"""GPU parity of the MoE FFN step (dyn_quant.moe) against the oracle: every
(token, expert) pair is the reference's split GEMV through w1 and w3, the
gated activation silu(a) * b rounded to FP16, then the split GEMV through w2;
the experts' outputs are added with the routing weights."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from dyn_quant import synth  # noqa: E402
from dyn_quant.moe import MoEFFN, MoERouting, moe_forward, silu_mul, silu_mul_pairs  # noqa: E402
from dq_testutil import check_y, dev, host  # noqa: E402
from test_moe_cpu import oracle_expert  # noqa: E402


def test_silu_mul_matches_numpy():
    rng = np.random.default_rng(1)
    a = (rng.standard_normal(4096) * 4).astype(np.float16)
    b = rng.standard_normal(4096).astype(np.float16)
    h = host(silu_mul(dev(a), dev(b)))
    af, bf = a.astype(np.float32), b.astype(np.float32)
    ref = (af / (np.float32(1) + np.exp(-af)) * bf).astype(np.float16)
    diff = np.abs(h.astype(np.float64) - ref.astype(np.float64))
    ulp = np.spacing(np.abs(ref.astype(np.float16))).astype(np.float64)
    assert (diff <= ulp).all()  # at most one FP16 ulp (exp differs by an FP32 ulp at most)


@pytest.mark.parametrize("E,D,F,T,K", [(4, 512, 1024, 8, 2), (8, 1024, 2048, 16, 2), (8, 4096, 14336, 16, 2)],
                         ids=["4x512x1024", "8x1024x2048", "mixtral-8x4096x14336"])
def test_moe_ffn_matches_oracle(E, D, F, T, K):
    """Every stage against the oracle given the GPU's own inputs to that stage
    (w1 and w3 on x, the gated activation on the GPU's a and b, w2 on the
    GPU's h: each a split GEMV at the split-GEMV tolerances), the combine
    against the FP32 weighted sum of the GPU's expert outputs, and the whole
    step against the oracle run end to end.  End to end the FP16 rounding of
    the intermediates a, b and h (and, rarely, an outlier decision near the
    threshold that follows from it) adds up, so the bound there is rel-L2
    5e-3."""
    import ctypes  # noqa: F401
    rng = np.random.default_rng(7)
    ex = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    mats = {}
    layer = MoEFFN(E, D, F)
    for e in range(E):
        w1, w3 = synth.weights(F, D, seed=10 + e), synth.weights(F, D, seed=20 + e)
        w2 = synth.weights(D, F, seed=30 + e)
        mats[e] = [(m, *O.quantize(m)) for m in (w1, w3, w2)]
        layer.load_expert(e, dev(w1), dev(w3), dev(w2))
    x = synth.activations(T, D, 0.02, seed=3)
    r_gpu = MoERouting(torch.from_numpy(ex), torch.from_numpy(w), E, device="cuda")
    r_cpu = MoERouting(torch.from_numpy(ex), torch.from_numpy(w), E, device="cpu")
    combined = np.zeros((T, D), np.float64)
    for e in range(E):
        rows = r_cpu.tokens.get(e)
        if rows is None:
            continue
        (w1, p1, s1, z1), (w3, p3, s3, z3), (w2, p2, s2, z2) = mats[e]
        xe = x[rows.numpy()]
        m = len(xe)
        ab = layer.gate_up(e, dev(xe))
        a, b = ab[:, :F], ab[:, F:]
        h = silu_mul_pairs(ab)
        assert torch.equal(h.view(torch.int16), silu_mul(a.contiguous(), b.contiguous()).view(torch.int16))
        y = layer.w2[str(e)](h).reshape(m, -1)
        a_h, b_h, h_h, y_h = host(a), host(b), host(h), host(y)
        for i in range(m):
            check_y(a_h[i], O.split_gemv(p1, s1, z1, w1, xe[i], 3.0)[0], what=f"expert {e} w1 row {i}")
            check_y(b_h[i], O.split_gemv(p3, s3, z3, w3, xe[i], 3.0)[0], what=f"expert {e} w3 row {i}")
            af, bf = a_h[i].astype(np.float32), b_h[i].astype(np.float32)
            ref_h = (af / (np.float32(1) + np.exp(-af)) * bf).astype(np.float16)
            assert (np.abs(h_h[i].astype(np.float64) - ref_h) <= np.spacing(np.abs(ref_h)).astype(np.float64)).all()
            check_y(y_h[i], O.split_gemv(p2, s2, z2, w2, h_h[i], 3.0)[0], what=f"expert {e} w2 row {i}")
        for i, t in enumerate(rows.tolist()):
            combined[t] += float(r_cpu.weight[e][i]) * y_h[i].astype(np.float64)
    out = host(layer(dev(x), r_gpu)).astype(np.float64)
    # the module's step equals the stages above, combined (FP32 sums, then FP16)
    assert np.abs(out - combined.astype(np.float16)).max() <= np.spacing(np.abs(combined).max().astype(np.float16))
    ref = moe_forward(torch.from_numpy(x), r_cpu, list(range(E)), lambda e, xe: oracle_expert(mats, e, xe),
                      torch.zeros(T, D), False).numpy().astype(np.float64)
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel <= 5e-3, rel


def test_moe_grouped_step_equals_the_expert_loop():
    """MoEFFN.forward runs the local experts through grouped batched calls
    (one for every w13, one for every w2); with at most 8 tokens on every
    expert those run the same kernels in the same geometry as the per-expert
    calls of moe_forward, so the step is bit-identical to the expert loop.
    (Between 2 and 8 tokens on every expert: a single token goes through the
    batch-1 kernel in the loop.)"""
    E, D, F, T, K = 8, 1024, 2048, 16, 2
    rng = np.random.default_rng(12)
    ex = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
    w = rng.random((T, K)).astype(np.float32)
    layer = MoEFFN(E, D, F)
    for e in range(E):
        layer.load_expert(e, dev(synth.weights(F, D, seed=40 + e)), dev(synth.weights(F, D, seed=50 + e)),
                          dev(synth.weights(D, F, seed=60 + e)))
    r = MoERouting(torch.from_numpy(ex), torch.from_numpy(w), E, device="cuda")
    assert all(2 <= r.count(e) <= 8 for e in range(E))
    x = dev(synth.activations(T, D, 0.02, seed=4))
    grouped = layer(x, r)
    loop = moe_forward(x, r, layer.local, layer.expert, torch.zeros(T, D, device="cuda"), False).to(torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(grouped.view(torch.int16), loop.view(torch.int16))
