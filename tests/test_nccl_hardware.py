"""Preflight on 2-4 real GPUs over NCCL and the peer-memory exchange; skipped with fewer than 2 GPUs
(never a Gloo run in disguise)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multi_gpu]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least two GPUs")
@pytest.mark.parametrize("grad_sync", ["peer", "nccl"])
def test_preflight_all_ranks(grad_sync):
    root = Path(__file__).resolve().parents[1]
    want = int(os.environ.get("THESEUS_TEST_RANKS", "4"))  # up to the visible GPUs
    ranks = max(2, min(want, torch.cuda.device_count()))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = os.environ | {"OMP_NUM_THREADS": "1", "TORCH_NCCL_ASYNC_ERROR_HANDLING": "1", "NCCL_NVLS_ENABLE": "0"}
    cmd = ["timeout", "-k", "30", "200", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={ranks}", "--master-addr=127.0.0.1", f"--master-port={port}",
           str(root / "check_nccl.py"), "--steps", "3", "--grad-sync", grad_sync]
    out = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=240)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert out.stdout.count('"status": "passed"') == 2
