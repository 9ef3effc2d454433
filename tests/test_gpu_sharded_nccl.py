"""Key-range sharded decode on 2 GPUs over NCCL (skipped with fewer than 2 GPUs).

Runs tests/multi/sharded_ranks.py under torchrun (127.0.0.1, a short process-group timeout, an
outer time limit, NVLS off): every rank's output must match the one-GPU decode over all keys,
for a single sequence (ShardedDecoder) and for a batch of sequences (BatchedShardedDecoder,
eager and captured in a CUDA graph with its NCCL all-gathers).
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).resolve().parent / "multi" / "sharded_ranks.py"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_sharded_decode_matches_one_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(WORKER)]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert res.stdout.count("allclose=True") == 2, res.stdout
