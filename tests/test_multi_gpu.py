"""Sharded step on two GPUs: two NCCL ranks run bench.py's step on their halves of
the heads, and rank 0 checks the gathered grad-grads against running every
head alone (they must be bit-identical: heads are independent and the kernels
are deterministic). Skipped with fewer than two GPUs."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_sharded_step_is_bit_identical():
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29517", "bench.py", "--gpus", "2",
           "--config", "c2", "--steps", "2", "--warmup", "3", "--verify"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["n_gpus"] == 2
    assert line["verify"]["bit_identical"], line["verify"]
