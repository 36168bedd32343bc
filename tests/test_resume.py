"""Whole runs under torchrun on CPU/Gloo: checkpoints, resume, export and the validation entry point.

The central property: a run interrupted at step boundaries and resumed from its checkpoints ends with the same
weights, optimizer state and reader cursors as the same run done in one go."""
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest
import torch
from safetensors.torch import load_file

from fixtures import make_config
from rwkv_theseus_b200.checkpoint import read_checkpoint

ROOT = Path(__file__).resolve().parents[1]
ENV = os.environ | {"OMP_NUM_THREADS": "1", "CUDA_VISIBLE_DEVICES": "", "TQDM_DISABLE": "0"}


def torchrun(script, ranks, *args, timeout=240, expect_ok=True):
    command = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
               f"--nproc_per_node={ranks}", str(ROOT / script), *map(str, args)]
    done = subprocess.run(command, env=ENV, cwd=ROOT, capture_output=True, text=True, timeout=timeout)
    if expect_ok:
        assert done.returncode == 0, done.stdout[-4000:] + done.stderr[-4000:]
    return done


def train(config_path, ranks=2, *extra, expect_ok=True):
    return torchrun("train.py", ranks, "--config", config_path, *extra, expect_ok=expect_ok)


def rewrite(path, cfg, **changes):
    cfg.update(changes)
    path.write_text(json.dumps(cfg))


def same_tensors(a, b, exact=True):
    assert a.keys() == b.keys()
    for key in a:
        if exact:
            assert torch.equal(a[key], b[key]), key
        else:
            torch.testing.assert_close(a[key], b[key], atol=1e-7, rtol=1e-6)


def test_interrupted_run_equals_uninterrupted_run(tmp_path):
    cfg, path = make_config(tmp_path, 2)
    rewrite(path, cfg, warmup_steps=1, constant_steps=0)
    train(path)
    rewrite(path, cfg, output=str(tmp_path / "pieces"))
    train(path, 2, "--stop-after", "1")
    train(path, 2, "--resume", tmp_path / "pieces", "--stop-after", "1")
    interim, meta, _ = read_checkpoint(tmp_path / "pieces")
    assert meta["step"] == 2 and not meta["complete"] and (interim / "COMMITTED").exists()
    assert not list((tmp_path / "pieces").glob(".*.tmp"))           # nothing left staged
    train(path, 2, "--resume", tmp_path / "pieces")
    whole, _, _ = read_checkpoint(tmp_path / "full")
    parts, final, _ = read_checkpoint(tmp_path / "pieces")
    assert final["complete"] and final["step"] == 3
    assert (tmp_path / "pieces" / "latest").read_text().strip() == parts.name
    same_tensors(load_file(str(whole / "migrated.safetensors")), load_file(str(parts / "migrated.safetensors")))
    opt_a = torch.load(whole / "optimizer.pt", weights_only=False)
    opt_b = torch.load(parts / "optimizer.pt", weights_only=False)
    for layer in final["order"]:
        state_a, state_b = opt_a[layer]["optimizer"]["state"], opt_b[layer]["optimizer"]["state"]
        for index in state_a:
            same_tensors(state_a[index], state_b[index])
        assert opt_a[layer]["scheduler"]["last_epoch"] == opt_b[layer]["scheduler"]["last_epoch"] == 3
    for rank in range(2):
        rank_a = torch.load(whole / "ranks" / f"rank_{rank:05d}.pt", weights_only=False)
        rank_b = torch.load(parts / "ranks" / f"rank_{rank:05d}.pt", weights_only=False)
        assert rank_a["reader"] == rank_b["reader"] and rank_a["runner"]["cursor"] == rank_b["runner"]["cursor"]
    # a complete run whose export never happened (interrupted after the final commit) only does the export
    shutil.rmtree(tmp_path / "pieces" / "converted")
    train(path, 2, "--resume", tmp_path / "pieces")
    assert json.loads((tmp_path / "pieces" / "converted" / "theseus.json").read_text())["format"] == 2
    report = torchrun("validate.py", 2, "--config", path, "--checkpoint", tmp_path / "pieces")
    results, _ = json.JSONDecoder().raw_decode(report.stdout[report.stdout.index("{"):])
    assert results["finite"] is True and results["original_teacher_kl"] >= 0


def test_resume_refuses_changed_settings_but_accepts_mutable_ones(tmp_path):
    cfg, path = make_config(tmp_path, 1)
    rewrite(path, cfg, original_teacher_kl=False, debug_input=False, stage_steps=4)
    train(path, 1, "--stop-after", "1")
    rewrite(path, cfg, chunk_tokens=2)
    refused = train(path, 1, "--resume", tmp_path / "full", expect_ok=False)
    assert refused.returncode != 0 and "Resume config changed: chunk_tokens" in refused.stderr
    rewrite(path, cfg, chunk_tokens=3, lr=5e-5, log_interval=3)
    train(path, 1, "--resume", tmp_path / "full", "--stop-after", "1")
    _, meta, _ = read_checkpoint(tmp_path / "full")
    assert meta["step"] == 2 and meta["config"]["lr"] == 5e-5


def test_sixteen_layers_on_four_ranks_export_and_reload(tmp_path):
    cfg, path = make_config(tmp_path, 16)
    rewrite(path, cfg, stage_steps=1, validation_chunks=1, original_teacher_kl=False, debug_input=False)
    train(path, 4)
    checkpoint, meta, delta = read_checkpoint(tmp_path / "full")
    assert meta["complete"] and meta["world"] == 4 and meta["order"] == list(range(1, 32, 2))
    assert set(delta) == set(meta["order"]) and all(len(params) == 23 for params in delta.values())
    out = tmp_path / "export"
    subprocess.run([sys.executable, str(ROOT / "export.py"), "--checkpoint", str(tmp_path / "full" / "latest"),
                    "--output", str(out)], check=True, capture_output=True, timeout=120, env=ENV, cwd=ROOT)
    record = json.loads((out / "theseus.json").read_text())
    assert record["layers"] == meta["order"] and record["base_fingerprint"] == meta["base_fingerprint"]
    from rwkv_theseus_b200.inference import load_export
    from rwkv_theseus_b200.models.hf_io import load_model
    base = load_model(tmp_path / "base", "cpu").state_dict()
    (tmp_path / "base").rename(tmp_path / "moved")                   # the export must not need the base
    runner = load_export(out, device="cpu")
    weights = runner.model.state_dict()
    for name, value in base.items():
        layer = int(name.split(".")[2]) if name.startswith("model.layers.") else None
        if layer not in meta["order"] or ".self_attn." not in name:
            assert torch.equal(weights[name], value), name
    for layer in meta["order"]:
        exported = weights[f"model.layers.{layer}.self_attn.core.receptance.weight"]
        assert torch.equal(exported, delta[layer]["receptance.weight"].to(exported.dtype))
    hidden = [runner.forward(torch.tensor([[5, 6, 7, 8]])) for _ in range(2)]
    assert all(torch.isfinite(h).all() for h in hidden) and runner.cache.cursor == 8


def test_epoch_mode_with_an_idle_rank_reads_every_token_once(tmp_path):
    cfg, path = make_config(tmp_path, 1)
    rewrite(path, cfg, training_mode="epoch", context_tokens=100, original_teacher_kl=False, validation_chunks=1)
    train(path, 4)   # three documents, four ranks: one rank contributes zero tokens every step
    done, meta, _ = read_checkpoint(tmp_path / "full")
    assert meta["complete"]
    events = [json.loads(line) for line in (tmp_path / "full" / "metrics.jsonl").read_text().splitlines()]
    trained = [e for e in events if e["event"] == "train"]
    assert len(trained) == meta["step"] and sum(e["tokens"] for e in trained) == 37
    cursors = [torch.load(done / "ranks" / f"rank_{r:05d}.pt", weights_only=False)["reader"] for r in range(4)]
    assert sum(c["consumed_tokens"] for c in cursors) == 37 and min(c["consumed_tokens"] for c in cursors) == 0
    rewrite(path, cfg, output=str(tmp_path / "again"))
    train(path, 4, "--stop-after", "1")
    train(path, 4, "--resume", tmp_path / "again")
    again, _, _ = read_checkpoint(tmp_path / "again")
    same_tensors(load_file(str(done / "migrated.safetensors")), load_file(str(again / "migrated.safetensors")),
                 exact=False)


@pytest.mark.parametrize("lanes", [2])
def test_lane_packed_epoch_resume_and_lane_change_after_completion(tmp_path, lanes):
    cfg, path = make_config(tmp_path, 1)
    rewrite(path, cfg, training_mode="epoch", micro_batch_size=lanes, context_tokens=7, original_teacher_kl=False,
            validation_chunks=1)
    train(path, 1, "--stop-after", "1")
    train(path, 1, "--resume", tmp_path / "full")
    done, meta, _ = read_checkpoint(tmp_path / "full")
    reader = torch.load(done / "ranks" / "rank_00000.pt", weights_only=False)["reader"]
    assert meta["complete"] and reader["reader_mode"] == "batched_epoch_v1" and reader["consumed_tokens"] == 37
    rewrite(path, cfg, micro_batch_size=4)   # allowed once the run is complete: only the export is redone
    train(path, 1, "--resume", tmp_path / "full")
