"""Row-sharded split GEMV on two GPUs: torch.distributed.run starts one rank
per GPU (NCCL); each rank runs the split GEMV kernel on its rows and the
output slices are all-gathered.  Needs at least two GPUs; skipped otherwise."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_row_sharded_two_gpus(tmp_path):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "sharded_worker.py"), str(tmp_path)]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    for r in range(2):
        res = json.load(open(tmp_path / f"rank{r}.json"))
        assert res["ok"], res
