"""Failure detection without any GPU fault: corrupted or partial checkpoints, a Gloo rank that fails
mid-run (the others end with an error instead of hanging), and step-phase profiling events."""
import json
import os
import shutil
import socket
import subprocess
import sys
from pathlib import Path

import pytest

from fixtures import make_config
from rwkv_theseus_b200.checkpoint import read_checkpoint

ROOT = Path(__file__).resolve().parents[1]


def _torchrun(script, ranks, *args, timeout=240, env=None):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(script), *map(str, args)]
    full_env = os.environ | {"OMP_NUM_THREADS": "1", "CUDA_VISIBLE_DEVICES": "", "PYTHONPATH": str(ROOT),
                             "TQDM_DISABLE": "1"} | (env or {})
    return subprocess.run(cmd, env=full_env, capture_output=True, text=True, timeout=timeout, cwd=ROOT)


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("ckpt")
    cfg, path = make_config(tmp, 2)
    out = _torchrun(ROOT / "train.py", 1, "--config", path, "--stop-after", 1)
    assert out.returncode == 0, out.stderr[-3000:]
    return Path(cfg["output"])


def test_uncommitted_checkpoint_is_rejected(trained, tmp_path):
    ckpt, _, _ = read_checkpoint(trained)
    copy = tmp_path / ckpt.name
    shutil.copytree(ckpt, copy)
    (copy / "COMMITTED").unlink()  # a crash between writing and committing
    with pytest.raises(ValueError, match="Not a committed checkpoint"):
        read_checkpoint(copy)


def test_truncated_weights_are_rejected(trained, tmp_path):
    ckpt, _, _ = read_checkpoint(trained)
    copy = tmp_path / ckpt.name
    shutil.copytree(ckpt, copy)
    data = (copy / "migrated.safetensors").read_bytes()
    (copy / "migrated.safetensors").write_bytes(data[: len(data) // 2])
    with pytest.raises(Exception):
        read_checkpoint(copy)


def test_latest_pointer_to_missing_directory_is_rejected(trained, tmp_path):
    root = tmp_path / "run"
    root.mkdir()
    (root / "latest").write_text("parallel_step_00000099\n")
    with pytest.raises((ValueError, FileNotFoundError)):
        read_checkpoint(root)


def test_failing_rank_ends_the_others_with_an_error():
    """Rank 1 raises before a collective; rank 0 must fail within the process-group timeout, not hang."""
    out = _torchrun(Path(__file__).with_name("dist_worker.py"), 2, "failing", timeout=180)
    assert out.returncode != 0
    assert "injected failure on rank 1" in out.stdout + out.stderr


def test_profile_events_report_step_phases(tmp_path):
    cfg, path = make_config(tmp_path, 2)
    out = _torchrun(ROOT / "train.py", 1, "--config", path, "--stop-after", 1, env={"THESEUS_PROFILE": "1"})
    assert out.returncode == 0, out.stderr[-3000:]
    events = [json.loads(line) for line in (Path(cfg["output"]) / "metrics.jsonl").read_text().splitlines()]
    prof = [e for e in events if e["event"] == "profile"]
    assert prof and prof[0]["teacher_ms"] > 0 and prof[0]["students_ms"] > 0
    assert {"student_01", "student_03", "update_01", "update_03"} <= set(prof[0]["phases_ms"])
