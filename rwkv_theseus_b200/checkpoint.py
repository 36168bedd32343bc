"""Atomic, rank-sharded checkpoints (format 2, ``parallel_layers_v1``).

On-disk layout (the reference's format, ``theseus/checkpoint.py:88-130``, kept so
that either project's tools read the other's checkpoints)::

    <output>/parallel_step_XXXXXXXX[_complete]/
        COMMITTED
        manifest.json          format, training_topology, stage, step, complete, order, config, world,
                               base/train/validation fingerprints, torch and transformers versions
        migrated.safetensors   "<layer>.<param>" fp32: the 23 TimeMix tensors of every migrated layer
        optimizer.pt           {layer: {"optimizer": AdamW state_dict, "scheduler": LambdaLR state_dict}}
        ranks/rank_XXXXX.pt    {"runner", "reader", "rng", "students": {layer: {shift, wkv}}}
    <output>/latest            name of the newest committed directory

A checkpoint becomes visible only when it is complete: every rank writes into a
hidden staging directory, the leader adds ``COMMITTED`` last, renames the
directory into place and swaps the ``latest`` pointer with an atomic replace.
Resuming is refused when the base weights, the data manifests, the layer order
or a config key outside ``MUTABLE_KEYS`` changed.
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
from torch.utils._pytree import tree_map

from .data import sha256_of_file

# Config keys that may change between a checkpoint and its resume (plus every ``wandb_*`` key).
MUTABLE_KEYS = frozenset({"output", "log_interval", "checkpoint_interval", "validation_interval",
                          "timeout_minutes", "lr", "warmup_steps", "constant_steps", "min_lr",
                          "fused_optimizer", "grad_sync", "student_graphs",
                          "overlap_students"})
# Values assumed for keys that older manifests do not carry.
_OLD_MANIFEST_DEFAULTS = {"training_mode": "sampled", "micro_batch_size": 1}


def cpu_tree(obj):
    """Detached CPU copies of every tensor in a nest of dicts, lists and tuples."""
    return tree_map(lambda leaf: leaf.detach().cpu().clone() if torch.is_tensor(leaf) else leaf, obj)


# Host generators saved with a checkpoint: key in the saved dict (the checkpoint layout), getter, setter.
_HOST_RNGS = (
    ("python", random.getstate, random.setstate),
    ("numpy", np.random.get_state, np.random.set_state),
    ("torch", torch.get_rng_state, lambda saved: torch.set_rng_state(saved.cpu())),
)


def rng_state():
    """Generator states of Python, NumPy, torch CPU and (when initialised) the current CUDA device."""
    saved = {key: get() for key, get, _ in _HOST_RNGS}
    saved["cuda"] = torch.cuda.get_rng_state() if torch.cuda.is_initialized() else None
    return saved


def restore_rng(saved):
    for key, _, put in _HOST_RNGS:
        put(saved[key])
    device_state = saved.get("cuda")
    if device_state is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state(device_state.cpu())


def model_fingerprint(path):
    """Identity of a base-model directory without reading its weights: the size and modification time of every
    ``*.safetensors`` shard and the SHA-256 of ``config.json`` / ``model.safetensors.index.json``, hashed as
    sorted JSON (the same record the reference writes into ``base_fingerprint``)."""
    root = Path(path)
    record = {}
    for shard in sorted(root.glob("*.safetensors")):
        info = shard.stat()
        record[shard.name] = [info.st_size, info.st_mtime_ns]
    for meta_file in ("config.json", "model.safetensors.index.json"):
        if (root / meta_file).exists():
            record[meta_file] = sha256_of_file(root / meta_file)
    return hashlib.sha256(json.dumps(record, sort_keys=True).encode()).hexdigest()


def split_delta(tensors):
    """``{"<layer>.<param>": t}`` -> ``{layer: {param: t}}``."""
    per_layer = {}
    for key, value in tensors.items():
        layer, param = key.split(".", 1)
        per_layer.setdefault(int(layer), {})[param] = value
    return per_layer


def resolve_checkpoint(path):
    """A committed checkpoint directory from the directory itself, its run root, or the root's ``latest`` file."""
    candidate = Path(path)
    if candidate.name == "latest" and candidate.is_file():
        candidate = candidate.parent / candidate.read_text().strip()
    elif not (candidate / "COMMITTED").exists() and (candidate / "latest").is_file():
        candidate = candidate / (candidate / "latest").read_text().strip()
    if not (candidate / "COMMITTED").exists():
        raise ValueError(f"Not a committed checkpoint: {candidate}")
    return candidate


def read_checkpoint(path):
    """(directory, manifest, {layer: {param: tensor}}) of a committed format-1 or format-2 checkpoint."""
    directory = resolve_checkpoint(path)
    manifest = json.loads((directory / "manifest.json").read_text())
    if manifest.get("format") not in (1, 2):
        raise ValueError("Unsupported checkpoint format")
    return directory, manifest, split_delta(load_file(str(directory / "migrated.safetensors")))


class _Staged:
    """One checkpoint directory being written: hidden while staged, renamed into place by ``commit``."""

    def __init__(self, root, step, complete):
        self.root = Path(root)
        self.name = f"parallel_step_{step:08d}" + ("_complete" if complete else "")
        self.final = self.root / self.name
        self.staging = self.root / f".{self.name}.tmp"

    def prepare(self):
        self.root.mkdir(parents=True, exist_ok=True)
        if self.staging.exists():
            shutil.rmtree(self.staging)
        (self.staging / "ranks").mkdir(parents=True)

    def commit(self):
        (self.staging / "COMMITTED").write_text("1\n")
        if self.final.exists():
            raise FileExistsError(f"Refusing to overwrite committed checkpoint {self.final}")
        os.replace(self.staging, self.final)
        pointer = self.root / ".latest.tmp"
        pointer.write_text(self.name + "\n")
        os.replace(pointer, self.root / "latest")


def _manifest(cfg, topo, step, complete, order, base_id):
    import transformers
    return {"format": 2, "training_topology": "parallel_layers_v1", "stage": 0, "step": step,
            "complete": complete, "order": order, "config": cfg, "world": topo.world,
            "base_fingerprint": base_id, "train_fingerprint": sha256_of_file(cfg["train_manifest"]),
            "validation_fingerprint": sha256_of_file(cfg["validation_manifest"]),
            "torch": torch.__version__, "transformers": transformers.__version__}


def save_checkpoint(topo, cfg, step, complete, order, runner, reader, base_id, students):
    """Collective: commit one checkpoint of every student; returns its directory."""
    target = _Staged(cfg["output"], step, complete)
    if topo.rank == topo.leader:
        target.prepare()
    topo.barrier()
    topo.join_grad_sync()
    for student in students.values():
        student.sync_state()  # complete fp32 masters and moments on every rank
    rank_file = {"runner": runner.state_dict(), "reader": None if reader is None else reader.state_dict(),
                 "rng": rng_state(), "students": {layer: s.state for layer, s in students.items()}}
    torch.save(cpu_tree(rank_file), target.staging / "ranks" / f"rank_{topo.rank:05d}.pt")
    if topo.rank == topo.leader:
        weights = {}
        optimizer = {}
        for layer, student in students.items():
            weights.update({f"{layer}.{param}": t.detach().cpu().contiguous()
                            for param, t in student.weights().items()})
            optimizer[layer] = {"optimizer": student.optimizer_state_dict(),
                                "scheduler": student.scheduler_state_dict()}
        save_file(weights, str(target.staging / "migrated.safetensors"))
        torch.save(cpu_tree(optimizer), target.staging / "optimizer.pt")
        manifest = _manifest(cfg, topo, step, complete, order, base_id)
        (target.staging / "manifest.json").write_text(json.dumps(manifest, indent=2))
    topo.barrier()
    if topo.rank == topo.leader:
        target.commit()
    topo.barrier()
    return target.final


def _changed_config_keys(saved, cfg, complete):
    allowed = set(MUTABLE_KEYS) | {key for key in cfg if key.startswith("wandb_")}
    if complete:
        allowed.add("micro_batch_size")
    changed = []
    for key in sorted(set(cfg) - allowed):
        before = saved.get(key, _OLD_MANIFEST_DEFAULTS.get(key))
        if cfg[key] != before:
            changed.append(key)
    return changed


def validate_resume(meta, cfg, topo, base_id, order):
    """Raise unless this job may continue the checkpoint described by `meta`."""
    if meta["base_fingerprint"] != base_id:
        raise ValueError("Base weights changed")
    if meta["order"] != order:
        raise ValueError("Migration layer order changed; start a new run.")
    for split in ("train", "validation"):
        if meta[f"{split}_fingerprint"] != sha256_of_file(cfg[f"{split}_manifest"]):
            raise ValueError(f"{split} manifest changed")
    changed = _changed_config_keys(meta["config"], cfg, meta["complete"])
    if changed:
        raise ValueError(f"Resume config changed: {changed[0]}")
    if meta["complete"]:
        return
    if meta.get("training_topology") not in ("local_branch_v1", "parallel_layers_v1"):
        raise ValueError("Old paired mid-stage checkpoints cannot resume; use a completed stage")
    if meta["world"] != topo.world:
        raise ValueError("Mid-stream resume needs identical rank topology")
