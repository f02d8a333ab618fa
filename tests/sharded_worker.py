"""One rank of the row-sharded GPU test (launched by tests/test_gpu_sharded.py
under torch.distributed.run, one process per GPU, NCCL).

Every rank builds the same seeded FP16 weight and activation, loads its row
slice into ShardedDynQuantLinear, runs forward with both gathers (the local
split GEMV kernel + an NCCL all-gather, and the kernel with the gather fused
over peer memory, three calls in a row) and checks every gathered y against
the oracle's full split GEMV within the split GEMV tolerances; the two
gathers must agree bit for bit.  Each rank writes one JSON result line to
<out_dir>/rank<r>.json.
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "dyn-quant_b200"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import ctypes as C  # noqa: E402
import datetime  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle as O  # noqa: E402
from dq_testutil import check_y  # noqa: E402
from dyn_quant import _lib, synth  # noqa: E402
from dyn_quant.sharded import ShardedDynQuantLinear, shard_rows  # noqa: E402

SHAPES = [(11008, 4096, 0.01), (1000, 1024, 0.03), (4096, 11008, 0.01)]


def main() -> None:
    out_dir = sys.argv[1]
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    results = []
    try:
        for i, (d_out, d_in, frac) in enumerate(SHAPES):
            w = synth.weights(d_out, d_in, seed=10 + i)
            packed, scales, zeros = O.quantize(w)
            lin = ShardedDynQuantLinear(d_in, d_out, 3.0)
            lin.load_weight(torch.from_numpy(w).to(dev))
            peer = ShardedDynQuantLinear(d_in, d_out, 3.0, gather="peer")
            peer.load_weight(torch.from_numpy(w).to(dev))
            for call in range(3):
                x = synth.activation(d_in, frac, seed=20 + 7 * i + call)
                xt = torch.from_numpy(x).to(dev)
                y = lin(xt)
                yp = peer(xt)
                torch.cuda.synchronize()
                same_gathers = bool(torch.equal(y.view(torch.int16), yp.view(torch.int16)))
                y = y.cpu().numpy()
                ref16, ref32, _ = O.split_gemv(packed, scales, zeros, w, x, 3.0)
                err = check_y(y, ref16, what=f"{d_out}x{d_in} call {call} rank {rank}")
                # every rank must hold the same gathered y, bit for bit
                yt = torch.from_numpy(y.copy()).to(dev)  # float16 (NCCL has no int16)
                y0 = yt.clone()
                dist.broadcast(y0, 0)
                same = bool(torch.equal(yt.view(torch.int16), y0.view(torch.int16)))
                r0, r1, per = shard_rows(d_out, world, rank)
                results.append({"shape": [d_out, d_in], "call": call, "rows": [r0, r1], "same_as_rank0": same,
                                "peer_same_as_nccl": same_gathers, **err})
            peer.close()
        err_word = C.c_uint32(0)
        _lib.check(_lib.lib().dq_read_device_error(C.byref(err_word), 0), "dq_read_device_error")
        ok = all(r["same_as_rank0"] and r["peer_same_as_nccl"] for r in results) and err_word.value == 0
        results.append({"device_error_word": err_word.value})
    except AssertionError as e:
        ok = False
        results.append({"error": str(e)})
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump({"rank": rank, "ok": ok, "results": results}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
