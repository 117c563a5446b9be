"""The row-sharded decode stack over NCCL on 2+ GPUs (skipped with fewer): every rank's logits
equal the unsharded CPU reference, eagerly and replayed from a CUDA graph."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_stack_matches_reference():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "stack_ranks.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0
