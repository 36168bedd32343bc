"""Multi-process CPU (Gloo) checks of the distributed plumbing (reference ``tests/test_distributed.py``)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(script, ranks, *args, timeout=180):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(script), *args]
    env = os.environ | {"OMP_NUM_THREADS": "1", "CUDA_VISIBLE_DEVICES": "", "PYTHONPATH": str(ROOT)}
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout, cwd=ROOT)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    return out.stdout


def test_token_weighted_gradient_matches_serial():
    _run(Path(__file__).with_name("dist_worker.py"), 4, "weighted")


def test_preflight_on_four_gloo_ranks():
    out = _run(ROOT / "check_nccl.py", 4, "--backend", "gloo", "--steps", "3")
    assert out.count('"status": "passed"') == 2


def test_mismatched_run_configuration_is_rejected():
    _run(Path(__file__).with_name("dist_worker.py"), 2, "mismatch")
