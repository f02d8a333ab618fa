"""Row sharding on CPU ranks (gloo, world size 2 and 3): the partition covers
every row once in whole 16-row blocks, and the gathered output of per-rank
oracle GEMVs on the row slices equals the oracle's full GEMV bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from dyn_quant import synth
from dyn_quant.sharded import ROW_BLOCK, ShardedDynQuantLinear, shard_rows


@pytest.mark.parametrize("d_out", [1, 16, 100, 4096, 11008, 28672])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition(d_out, world):
    seen = np.zeros(d_out, np.int32)
    heights = set()
    for r in range(world):
        r0, r1, per = shard_rows(d_out, world, r)
        heights.add(per)
        assert per % ROW_BLOCK == 0 and r1 - r0 <= per
        assert r0 % ROW_BLOCK == 0 or r0 == d_out
        seen[r0:r1] += 1
    assert len(heights) == 1 and (seen == 1).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, d_out, d_in, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = synth.weights(d_out, d_in, seed=3)
        x = synth.activation(d_in, 0.02, seed=4)
        packed, scales, zeros = O.quantize(w)
        r0, r1, _ = shard_rows(d_out, world, rank)

        def local(_x):
            if r1 <= r0:
                return torch.empty(0, dtype=torch.float16)
            y16, _, _ = O.split_gemv(packed[r0:r1], scales[r0:r1], zeros[r0:r1], w[r0:r1], x, 3.0)
            return torch.from_numpy(y16)

        lin = ShardedDynQuantLinear(d_in, d_out, 3.0, local_gemv=local)
        y = lin(torch.from_numpy(x)).numpy()
        full, _, _ = O.split_gemv(packed, scales, zeros, w, x, 3.0)
        q.put((rank, bool(np.array_equal(y.view(np.uint16), full.view(np.uint16)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,d_out,d_in", [(2, 100, 512), (3, 257, 1024), (2, 48, 256)])
def test_sharded_gather_matches_full_gemv(world, d_out, d_in):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, d_out, d_in, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok in results), results
