"""GPU, two or more devices: the N-sharded GEMM (column shards per rank,
NCCL all-gather of Y over NVLink) matches the unsharded result and the
oracle.  Runs one process per GPU through torch.distributed.run; skipped on
single-GPU machines (the host logic is covered by test_sharding_cpu.py)."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_n_sharded_gemm_allgather_two_gpus(cuda):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    worker = Path(__file__).resolve().parent / "_mgpu_worker.py"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={min(n, 2)}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(worker)]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(p.stdout[-4000:])
    assert p.returncode == 0, p.stderr[-4000:]
