"""End-to-end torchrun runs on CPU/Gloo: train, resume bit-exactly, export, validate."""
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import torch
from safetensors.torch import load_file

from fixtures import make_config
from rwkv_theseus_b200.checkpoint import read_checkpoint

ROOT = Path(__file__).resolve().parents[1]
ENV = os.environ | {"OMP_NUM_THREADS": "1", "CUDA_VISIBLE_DEVICES": "", "TQDM_DISABLE": "0"}


def torchrun(script, ranks, *args, timeout=240):
    command = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
               f"--nproc_per_node={ranks}", str(ROOT / script), *map(str, args)]
    result = subprocess.run(command, env=ENV, cwd=ROOT, capture_output=True, text=True, timeout=timeout)
    assert result.returncode == 0, result.stdout[-4000:] + result.stderr[-4000:]
    return result


def launch(config, ranks=2, extra=()):
    return torchrun("train.py", ranks, "--config", config, *extra)


def test_parallel_midstream_and_complete_resume(tmp_path):
    cfg, path = make_config(tmp_path, 2)
    cfg.update(warmup_steps=1, constant_steps=0)
    path.write_text(json.dumps(cfg))
    launch(path)
    cfg["output"] = str(tmp_path / "resumed")
    path.write_text(json.dumps(cfg))
    launch(path, extra=("--stop-after", "1"))
    launch(path, extra=("--resume", tmp_path / "resumed", "--stop-after", "2"))
    _, mid, _ = read_checkpoint(tmp_path / "resumed")
    assert mid["step"] == 3 and mid["complete"]
    shutil.rmtree(tmp_path / "resumed" / "converted")   # interrupted after commit, before export
    launch(path, extra=("--resume", tmp_path / "resumed"))
    af, _, _ = read_checkpoint(tmp_path / "full")
    bf, _, _ = read_checkpoint(tmp_path / "resumed")
    a, b = load_file(str(af / "migrated.safetensors")), load_file(str(bf / "migrated.safetensors"))
    assert a.keys() == b.keys()
    for key in a:
        torch.testing.assert_close(a[key], b[key], atol=0, rtol=0)
    for rank in range(2):
        sa = torch.load(af / "ranks" / f"rank_{rank:05d}.pt", weights_only=False)
        sb = torch.load(bf / "ranks" / f"rank_{rank:05d}.pt", weights_only=False)
        assert sa["reader"] == sb["reader"]
        assert sa["runner"]["cursor"] == sb["runner"]["cursor"]
    result = torchrun("validate.py", 2, "--config", path, "--checkpoint", bf)
    assert "original_teacher_kl" in result.stdout


def test_four_rank_all_sixteen_stages_and_export(tmp_path):
    cfg, path = make_config(tmp_path, 16)
    cfg.update(stage_steps=1, validation_chunks=1, original_teacher_kl=False, debug_input=False)
    path.write_text(json.dumps(cfg))
    launch(path, ranks=4)
    checkpoint, meta, delta = read_checkpoint(tmp_path / "full")
    assert meta["complete"] and meta["training_topology"] == "parallel_layers_v1" and len(delta) == 16
    assert meta["order"] == list(range(1, 32, 2))
    out = tmp_path / "export"
    subprocess.run([sys.executable, str(ROOT / "export.py"), "--checkpoint", str(checkpoint), "--output", str(out)],
                   check=True, capture_output=True, timeout=120, env=ENV, cwd=ROOT)
    from rwkv_theseus_b200.inference import load_export
    (tmp_path / "base").rename(tmp_path / "base_hidden")
    runner = load_export(out, device="cpu")
    assert (out / "model.safetensors").exists() and not (out / "migrated.safetensors").exists()
    opt = torch.load(checkpoint / "optimizer.pt", weights_only=False)
    assert set(opt) == set(meta["order"])
    for _ in range(2):
        assert torch.isfinite(runner.forward(torch.tensor([[1, 2, 3]]))).all()
    assert runner.cache.cursor == 6
    from rwkv_theseus_b200.models.hf_io import load_model
    base = load_model(tmp_path / "base_hidden", "cpu")
    actual = runner.model.state_dict()
    for name, value in base.state_dict().items():
        if not any(name.startswith(f"model.layers.{layer}.self_attn.") for layer in meta["order"]):
            torch.testing.assert_close(actual[name], value, atol=0, rtol=0)


def test_single_rank_local_training(tmp_path):
    cfg, path = make_config(tmp_path, 1)
    cfg.update(stage_steps=2, validation_interval=1)
    path.write_text(json.dumps(cfg))
    result = launch(path, ranks=1)
    assert "Parallel migration (1 layers)" in result.stderr
    assert "sum_loss=" in result.stderr and "mean_cos=" in result.stderr
    _, meta, delta = read_checkpoint(tmp_path / "full")
    assert meta["world"] == 1 and meta["complete"] and len(delta) == 1


def test_epoch_uneven_ranks_exact_coverage_and_resume(tmp_path):
    cfg, path = make_config(tmp_path, 1)
    cfg.update(training_mode="epoch", context_tokens=100, stage_steps=1, original_teacher_kl=False,
               validation_chunks=1)
    path.write_text(json.dumps(cfg))
    launch(path, ranks=4)   # three documents on four ranks: one rank is empty all epoch
    complete, meta, _ = read_checkpoint(tmp_path / "full")
    assert meta["complete"] and meta["step"] == 3
    events = [json.loads(line) for line in (tmp_path / "full/metrics.jsonl").read_text().splitlines()]
    assert sum(e["tokens"] for e in events if e["event"] == "train") == 37
    consumed = sum(torch.load(complete / "ranks" / f"rank_{r:05d}.pt", weights_only=False)["reader"]["consumed_tokens"]
                   for r in range(4))
    assert consumed == 37
    cfg["output"] = str(tmp_path / "resumed")
    path.write_text(json.dumps(cfg))
    launch(path, ranks=4, extra=("--stop-after", "1"))
    launch(path, ranks=4, extra=("--resume", tmp_path / "resumed"))
    resumed, _, _ = read_checkpoint(tmp_path / "resumed")
    a = load_file(str(complete / "migrated.safetensors"))
    b = load_file(str(resumed / "migrated.safetensors"))
    for key in a:
        torch.testing.assert_close(a[key], b[key], atol=1e-7, rtol=1e-6)


def test_batched_epoch_single_rank_training_and_resume(tmp_path):
    cfg, path = make_config(tmp_path, 1)
    cfg.update(training_mode="epoch", micro_batch_size=2, context_tokens=7, original_teacher_kl=False,
               validation_interval=0, validation_chunks=1)
    path.write_text(json.dumps(cfg))
    launch(path, ranks=1, extra=("--stop-after", "1"))
    launch(path, ranks=1, extra=("--resume", tmp_path / "full"))
    checkpoint, meta, _ = read_checkpoint(tmp_path / "full")
    assert meta["complete"]
    state = torch.load(checkpoint / "ranks" / "rank_00000.pt", weights_only=False)
    assert state["reader"]["consumed_tokens"] == 37
    cfg["micro_batch_size"] = 4
    path.write_text(json.dumps(cfg))
    launch(path, ranks=1, extra=("--resume", tmp_path / "full"))
