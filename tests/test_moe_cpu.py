"""The MoE layer's routing and distribution logic on CPU ranks (gloo): the
per-expert token lists of a top-k routing, and the sum over ranks of the
ranks' experts equals the single-rank result (experts are oracle split-GEMV
FFNs on small shapes)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from dyn_quant import synth
from dyn_quant.moe import MoERouting, moe_forward

E, D, F, T, K = 4, 256, 512, 8, 2


def _routing(seed=5):
    rng = np.random.default_rng(seed)
    ex = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    return torch.from_numpy(ex), torch.from_numpy(w)


def _experts():
    mats = {}
    for e in range(E):
        w1, w3 = synth.weights(F, D, seed=10 + e), synth.weights(F, D, seed=20 + e)
        w2 = synth.weights(D, F, seed=30 + e)
        mats[e] = [(w, *O.quantize(w)) for w in (w1, w3, w2)]
    return mats


def oracle_expert(mats, e, xe):
    """Expert e on the rows of xe (float16 CPU tensor), the reference's split GEMV per row."""
    out = []
    for x in xe.numpy():
        (w1, p1, s1, z1), (w3, p3, s3, z3), (w2, p2, s2, z2) = mats[e]
        a = O.split_gemv(p1, s1, z1, w1, x, 3.0)[0].astype(np.float32)
        b = O.split_gemv(p3, s3, z3, w3, x, 3.0)[0].astype(np.float32)
        h = (a / (1.0 + np.exp(-a)) * b).astype(np.float16)
        out.append(O.split_gemv(p2, s2, z2, w2, h, 3.0)[0])
    return torch.from_numpy(np.stack(out))


def test_routing_lists():
    ex, w = _routing()
    r = MoERouting(ex, w, E, device="cpu")
    seen = {}
    for e in range(E):
        for i, t in enumerate(r.tokens.get(e, torch.empty(0, dtype=torch.int32)).tolist()):
            slot = ex[t].tolist().index(e)
            assert r.weight[e][i].item() == w[t, slot].item()
            seen[(t, e)] = 1
    assert len(seen) == T * K
    with pytest.raises(ValueError):
        MoERouting(torch.tensor([[0, 0]]), torch.ones(1, 2), E, device="cpu")
    with pytest.raises(ValueError):
        MoERouting(torch.tensor([[0, E]]), torch.ones(1, 2), E, device="cpu")


def test_stacked_rows_follow_the_expert_order():
    """The grouped step's row gather: the experts' token lists one after
    another, in the order asked for, with their counts; cached per order."""
    ex, w = _routing()
    r = MoERouting(ex, w, E, device="cpu")
    order = [e for e in (2, 0, 3, 1) if r.count(e)]
    rows, counts = r.stacked(order)
    assert counts == [r.count(e) for e in order]
    assert rows.tolist() == sum((r.tokens64[e].tolist() for e in order), [])
    assert r.stacked(order)[0] is rows
    assert r.stacked(list(reversed(order)))[0] is not rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mats = _experts()
        ex, w = _routing()
        r = MoERouting(ex, w, E, device="cpu")
        x = torch.from_numpy(synth.activations(T, D, 0.02, seed=3))
        local = [e for e in range(E) if e % world == rank]
        out = moe_forward(x, r, local, lambda e, xe: oracle_expert(mats, e, xe), torch.zeros(T, D), True)
        full = moe_forward(x, r, list(range(E)), lambda e, xe: oracle_expert(mats, e, xe), torch.zeros(T, D), False)
        q.put((rank, float((out - full).abs().max() / full.abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_experts_over_ranks_sum_to_single_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 1e-6 for _, err in res), res
