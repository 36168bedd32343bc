"""Atomic, rank-sharded checkpoints (format 2, ``parallel_layers_v1``).

Layout (reference ``theseus/checkpoint.py:88-130``)::

    <output>/parallel_step_XXXXXXXX[_complete]/
        COMMITTED
        manifest.json          format, topology, step, order, config, world, fingerprints, versions
        migrated.safetensors   "<layer>.<param>" fp32, the 23 TimeMix tensors per layer
        optimizer.pt           {layer: {"optimizer": AdamW state_dict, "scheduler": LambdaLR state_dict}}
        ranks/rank_XXXXX.pt    {"runner", "reader", "rng", "students": {layer: {shift, wkv}}}
    <output>/latest            name of the newest committed directory

Commit protocol: leader creates ``.<name>.tmp``; barrier; every rank writes its
own file; leader writes weights, optimizer and manifest; barrier; leader writes
``COMMITTED``, renames the directory into place and atomically replaces
``latest``; barrier. Resume is guarded by base/manifest fingerprints, the
layer order and the non-mutable config keys.
"""
import hashlib
import json
import os
import random
import shutil
from pathlib import Path

import numpy as np
import torch
from safetensors.torch import load_file, save_file

from .data import digest_file

MUTABLE_KEYS = {"output", "log_interval", "checkpoint_interval", "validation_interval", "timeout_minutes",
                "lr", "warmup_steps", "constant_steps", "min_lr", "fused_optimizer", "grad_sync", "student_graphs"}


def cpu_tree(obj):
    if torch.is_tensor(obj):
        return obj.detach().cpu().clone()
    if isinstance(obj, dict):
        return {k: cpu_tree(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [cpu_tree(v) for v in obj]
    if isinstance(obj, tuple):
        return tuple(cpu_tree(v) for v in obj)
    return obj


def rng_state():
    return {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state() if torch.cuda.is_initialized() else None}


def restore_rng(state):
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"].cpu())
    if state["cuda"] is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state(state["cuda"].cpu())


def model_fingerprint(path):
    """Hash of shard sizes/mtimes plus config/index content (cheap, no weight read)."""
    path = Path(path)
    records = {p.name: (p.stat().st_size, p.stat().st_mtime_ns) for p in sorted(path.glob("*.safetensors"))}
    for p in (path / "config.json", path / "model.safetensors.index.json"):
        if p.exists():
            records[p.name] = digest_file(p)
    return hashlib.sha256(json.dumps(records, sort_keys=True).encode()).hexdigest()


def split_delta(tensors):
    out = {}
    for key, value in tensors.items():
        layer, name = key.split(".", 1)
        out.setdefault(int(layer), {})[name] = value
    return out


def resolve_checkpoint(path):
    path = Path(path)
    if path.name == "latest":
        path = path.parent / path.read_text().strip()
    elif not (path / "COMMITTED").exists() and (path / "latest").exists():
        path = path / (path / "latest").read_text().strip()
    if not (path / "COMMITTED").exists():
        raise ValueError(f"Not a committed checkpoint: {path}")
    return path


def read_checkpoint(path):
    path = resolve_checkpoint(path)
    meta = json.loads((path / "manifest.json").read_text())
    if meta["format"] not in (1, 2):
        raise ValueError("Unsupported checkpoint format")
    return path, meta, split_delta(load_file(str(path / "migrated.safetensors")))


def save_checkpoint(topo, cfg, step, complete, order, runner, reader, base_id, students):
    """Commit one parallel-layer checkpoint; returns its final directory."""
    root = Path(cfg["output"])
    name = f"parallel_step_{step:08d}" + ("_complete" if complete else "")
    final, temp = root / name, root / f".{name}.tmp"
    if topo.rank == topo.leader:
        root.mkdir(parents=True, exist_ok=True)
        if temp.exists():
            shutil.rmtree(temp)
        (temp / "ranks").mkdir(parents=True)
    topo.barrier()
    topo.join_grad_sync()
    for s in students.values():
        s.sync_state()
    local = {"runner": runner.state_dict(), "reader": reader.state_dict() if reader else None, "rng": rng_state(),
             "students": {layer: s.state for layer, s in students.items()}}
    torch.save(cpu_tree(local), temp / "ranks" / f"rank_{topo.rank:05d}.pt")
    if topo.rank == topo.leader:
        weights = {f"{layer}.{k}": v.detach().cpu().contiguous()
                   for layer, s in students.items() for k, v in s.weights().items()}
        save_file(weights, str(temp / "migrated.safetensors"))
        optim = {layer: {"optimizer": s.optimizer_state_dict(), "scheduler": s.scheduler_state_dict()}
                 for layer, s in students.items()}
        torch.save(cpu_tree(optim), temp / "optimizer.pt")
        import transformers
        meta = {"format": 2, "training_topology": "parallel_layers_v1", "stage": 0, "step": step,
                "complete": complete, "order": order, "config": cfg, "world": topo.world,
                "base_fingerprint": base_id, "train_fingerprint": digest_file(cfg["train_manifest"]),
                "validation_fingerprint": digest_file(cfg["validation_manifest"]),
                "torch": torch.__version__, "transformers": transformers.__version__}
        (temp / "manifest.json").write_text(json.dumps(meta, indent=2))
    topo.barrier()
    if topo.rank == topo.leader:
        (temp / "COMMITTED").write_text("1\n")
        if final.exists():
            raise FileExistsError(f"Refusing to overwrite committed checkpoint {final}")
        os.replace(temp, final)
        pointer = root / ".latest.tmp"
        pointer.write_text(name + "\n")
        os.replace(pointer, root / "latest")
    topo.barrier()
    return final


def validate_resume(meta, cfg, topo, base_id, order):
    if meta["base_fingerprint"] != base_id:
        raise ValueError("Base weights changed")
    if meta["order"] != order:
        raise ValueError("Migration layer order changed; start a new run.")
    for name in ("train", "validation"):
        if meta[name + "_fingerprint"] != digest_file(cfg[name + "_manifest"]):
            raise ValueError(f"{name} manifest changed")
    mutable = set(MUTABLE_KEYS)
    if meta["complete"]:
        mutable.add("micro_batch_size")
    for key in cfg.keys() - mutable - {k for k in cfg if k.startswith("wandb_")}:
        default = "sampled" if key == "training_mode" else 1 if key == "micro_batch_size" else None
        if key in ("lora_rank", "gate_lora_rank") and key not in meta["config"]:
            default = None
        if cfg[key] != meta["config"].get(key, default):
            raise ValueError(f"Resume config changed: {key}")
    if not meta["complete"]:
        if meta.get("training_topology") not in {"local_branch_v1", "parallel_layers_v1"}:
            raise ValueError("Old paired mid-stage checkpoints cannot resume; use a completed stage")
        if meta["world"] != topo.world:
            raise ValueError("Mid-stream resume needs identical rank topology")
