"""Strict JSON run configuration.

The key set, the defaults and what is accepted follow the reference's
``configs/train.json`` contract (``theseus/config.py:4-75``): a supplied JSON
object overrides the defaults, unknown keys are an error, counts must be
positive integers, ``cosine_weight`` must stay 0 (parallel migration optimises
NMSE only) and the four path keys are made absolute.

This module states that contract as data: every key has a ``Field`` (its
default and the kind of value it takes), and the constraints between keys are
a list of named rules checked in order. A config therefore fails with the
message of the first key, then the first rule, that it breaks.

Keys added on top of the reference schema (defaults keep reference behaviour,
so a reference ``configs/train.json`` loads unchanged):

* ``lora_rank`` / ``gate_lora_rank``: TimeMix LoRA widths; ``None`` derives them
  from the model width as the reference does (``theseus/timemix.py:35-36``).
* ``fused_optimizer``: flat-buffer fused clip + AdamW kernels on CUDA (default);
  ``False`` uses ``torch.optim.AdamW``.
* ``grad_sync``: multi-GPU gradient path of the fused optimizer, ``"peer"``
  (NVLink peer-memory exchange with sharded AdamW) or ``"nccl"`` (all-reduce,
  then the full update on every rank, as the reference does).
* ``student_graphs``: replay each fused student micro-step as a CUDA graph.
* ``overlap_students``: run the students' micro-steps on a CUDA stream of their
  own, each starting once the teacher forward has produced its layer's capture
  (beside the rest of the teacher forward).
"""
import json
from dataclasses import dataclass
from pathlib import Path


@dataclass(frozen=True)
class Field:
    default: object
    kind: str = "any"        # any | count | nonneg_int | bool | optional_count | path | str
    choices: tuple = ()


SCHEMA = {
    # paths and model geometry
    "model": Field("../Qwen3.8-27B", "path"),
    "train_manifest": Field("data/train/manifest.json", "path"),
    "validation_manifest": Field("data/val/manifest.json", "path"),
    "output": Field("runs/theseus_parallel", "path"),
    "expected_attention_layers": Field(16, "count"),
    "head_size": Field(64, "count"),
    "backend": Field("cuda", choices=("cuda", "reference")),
    "seed": Field(42),
    # data and schedule
    "chunk_tokens": Field(256, "count"),
    "context_tokens": Field(4096, "count"),
    "stage_steps": Field(1000),
    "training_mode": Field("epoch", choices=("epoch", "sampled")),
    "grad_accum_steps": Field(1, "count"),
    "micro_batch_size": Field(1, "count"),
    # optimiser
    "lr": Field(1e-4),
    "betas": Field([0.9, 0.999]),
    "adam_eps": Field(1e-8),
    "weight_decay": Field(0.01),
    "clip_norm": Field(1.0),
    "warmup_steps": Field(300, "nonneg_int"),
    "constant_steps": Field(3000, "nonneg_int"),
    "min_lr": Field(3e-6),
    # loss, validation, logging
    "cosine_weight": Field(0.0),
    "loss_epsilon": Field(1e-6),
    "checkpoint_interval": Field(3000),
    "validation_interval": Field(100),
    "validation_chunks": Field(8, "count"),
    "log_interval": Field(10, "count"),
    "original_teacher_kl": Field(False),
    "kl_token_block": Field(16, "count"),
    "debug_input": Field(False),
    "wandb_mode": Field("disabled", choices=("disabled", "offline", "online")),
    "wandb_project": Field("RWKV-Theseus", "str"),
    "wandb_entity": Field(None),
    "wandb_name": Field(None),
    # process groups
    "distributed_backend": Field("nccl", choices=("nccl", "gloo")),
    "timeout_minutes": Field(60),
    # extensions of this implementation
    "lora_rank": Field(None, "optional_count"),
    "gate_lora_rank": Field(None, "optional_count"),
    "fused_optimizer": Field(True, "bool"),
    "grad_sync": Field("peer", choices=("peer", "nccl")),
    "student_graphs": Field(True, "bool"),
    "overlap_students": Field(True, "bool"),
}

DEFAULTS = {name: field.default for name, field in SCHEMA.items()}


def _is_int(value):
    return type(value) is int


def _field_error(name, field, value):
    """Message for a value that does not fit its field, or None."""
    if field.choices and value not in field.choices:
        if name in ("backend", "distributed_backend"):
            return "Unsupported backend"
        head, last = field.choices[:-1], field.choices[-1]
        return f"{name} must be {', '.join(head)} or {last}"
    if field.kind == "count" and not (_is_int(value) and value > 0):
        return f"{name} must be a positive integer"
    if field.kind == "nonneg_int" and not (_is_int(value) and value >= 0):
        return f"{name} must be a nonnegative integer"
    if field.kind == "optional_count" and value is not None and not (_is_int(value) and value > 0):
        return f"{name} must be null or a positive integer"
    if field.kind == "bool" and not isinstance(value, bool):
        return f"{name} must be a boolean"
    if field.kind == "str" and not (isinstance(value, str) and value.strip()):
        return f"{name} must be nonempty"
    return None


def _stage_list(cfg):
    steps = cfg["stage_steps"]
    return steps if isinstance(steps, list) else [steps]


# Cross-key rules: (predicate that holds for a valid config, message).
RULES = (
    (lambda c: c["context_tokens"] >= c["chunk_tokens"], "context_tokens must be >= chunk_tokens"),
    (lambda c: c["micro_batch_size"] == 1 or c["training_mode"] == "epoch",
     "micro_batch_size > 1 currently requires training_mode=epoch"),
    (lambda c: c["training_mode"] != "sampled" or (
        len(_stage_list(c)) in (1, c["expected_attention_layers"]) and min(_stage_list(c)) >= 1),
     "stage_steps must be positive or a per-stage list"),
    (lambda c: len(set(_stage_list(c))) == 1, "Parallel migration requires equal stage_steps for all layers"),
    (lambda c: c["cosine_weight"] == 0, "Parallel migration optimizes NMSE only; cosine_weight must be zero"),
    (lambda c: c["lr"] > 0 and c["clip_norm"] > 0, "Invalid optimization configuration"),
    (lambda c: 0 <= c["min_lr"] <= c["lr"], "min_lr must be between zero and lr"),
    (lambda c: c["checkpoint_interval"] >= 0, "checkpoint_interval must be >= 0"),
    (lambda c: c["validation_interval"] >= 0, "validation_interval must be >= 0"),
    (lambda c: c["backend"] != "cuda" or 2 <= c["head_size"] <= 128, "CUDA supports head_size in 2..128"),
    (lambda c: not (c["backend"] == "cuda" and c["distributed_backend"] == "gloo"),
     "Gloo is CPU smoke-test mode; choose backend=reference"),
    (lambda c: c["loss_epsilon"] > 0, "Invalid loss configuration"),
)


def make_config(supplied):
    """Validate a dict of overrides against the schema and return the complete, path-resolved config."""
    unknown = set(supplied) - set(SCHEMA)
    if unknown:
        raise ValueError(f"Unknown config keys: {unknown}")
    cfg = {name: supplied.get(name, field.default) for name, field in SCHEMA.items()}
    for name, field in SCHEMA.items():
        problem = _field_error(name, field, cfg[name])
        if problem:
            raise ValueError(problem)
    for holds, message in RULES:
        if not holds(cfg):
            raise ValueError(message)
    for name, field in SCHEMA.items():
        if field.kind == "path":
            cfg[name] = str(Path(cfg[name]).resolve())
    return cfg


def load_config(path):
    """Read a JSON object from `path` and return the validated config."""
    return make_config(json.loads(Path(path).read_text()))


def steps_for(cfg, stage):
    """Step budget of one stage; a one-element list applies to every stage."""
    budget = _stage_list(cfg)
    return budget[stage] if len(budget) > 1 else budget[0]
