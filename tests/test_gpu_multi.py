"""Multi-GPU parity (batch sharding and context parallelism over NCCL).

Runs tests/multi_gpu_worker.py under torchrun with one rank per visible GPU
(at most 8); skipped when fewer than two GPUs are visible.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_batch_sharding_and_context_parallel_on_all_gpus():
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs at least two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [
        "timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
        f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29531",
        str(ROOT / "tests" / "multi_gpu_worker.py"),
    ]
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    assert proc.stdout.count(" OK") == n, proc.stdout[-4000:]
