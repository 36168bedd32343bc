"""Checkpoint-level operations behind the ``export.py`` and ``validate.py`` entry points.

Both start from a committed checkpoint (``checkpoint.read_checkpoint``) and the
base model it was trained from, which must be unchanged (fingerprint check).

* ``export_checkpoint`` (reference ``export.py:8-23``): a complete checkpoint ->
  the base model with every trained student installed in place of its attention,
  written as export format 2 (``inference.save_export``). Incomplete
  checkpoints are refused.
* ``validate_checkpoint`` (reference ``validate.py:13-48``): which validation
  runs depends on what the checkpoint holds: a complete parallel checkpoint is
  validated as an assembled model, an incomplete one layer by layer
  (teacher-forced), and a legacy sequential checkpoint with the single-stage
  validation of its current stage.
"""
import json

from .checkpoint import model_fingerprint, read_checkpoint
from .inference import save_export
from .models.hf_io import load_model
from .models.runner import Capture, Runner, install
from .validation import validate, validate_composition, validate_parallel


def _require_same_base(cfg, meta, message):
    if model_fingerprint(cfg["model"]) != meta["base_fingerprint"]:
        raise ValueError(message)


def _base_with_students(cfg, delta, layers, device):
    model = load_model(cfg["model"], device)
    for layer in layers:
        install(model, layer, cfg, delta[layer])
    return model


def export_checkpoint(checkpoint, output):
    """Write the export of a complete checkpoint to `output`; returns `output`."""
    directory, meta, delta = read_checkpoint(checkpoint)
    if not meta["complete"] or set(delta) != set(meta["order"]):
        raise ValueError("Final export requires all layers to have completed training")
    cfg = meta["config"]
    _require_same_base(cfg, meta, "Base weights changed")
    model = _base_with_students(cfg, delta, meta["order"], "cpu")
    save_export(model, output, cfg, meta["order"], meta["base_fingerprint"], checkpoint=directory)
    return output


def _parallel_students(topo, cfg, model, meta, delta):
    from .stage import Student
    students = {layer: Student(model.config, layer, cfg, topo, delta[layer]) for layer in meta["order"]}
    captures = {layer: Capture(model.model.layers[layer].self_attn) for layer in meta["order"]}
    try:
        return validate_parallel(topo, cfg, Runner(model), students, captures)
    finally:
        for capture in captures.values():
            capture.close()


def _sequential_stage(topo, cfg, model, meta, delta):
    done, current = meta["order"][:meta["stage"]], meta["order"][meta["stage"]]
    for layer in done:
        install(model, layer, cfg, delta[layer])
    install(model, current, cfg, delta[current], trainable=True, retain_teacher=True)
    model.requires_grad_(False)
    return validate(topo, cfg, Runner(model), current)


def validate_checkpoint(cfg, checkpoint):
    """Collective over the launched ranks; the leader prints the results as JSON. Returns them."""
    from .parallel.topology import Topology
    topo = Topology(cfg["distributed_backend"], cfg["timeout_minutes"])
    topo.assert_same({"config": cfg, "checkpoint": checkpoint}, "validation configuration")
    _, meta, delta = read_checkpoint(checkpoint)
    _require_same_base(cfg, meta, "Validation base differs from training")
    if meta.get("training_topology") != "parallel_layers_v1":
        results = _sequential_stage(topo, cfg, load_model(cfg["model"], topo.device), meta, delta)
    elif meta["complete"]:
        assembled = _base_with_students(cfg, delta, meta["order"], topo.device)
        results = validate_composition(topo, cfg, Runner(assembled))
    else:
        results = _parallel_students(topo, cfg, load_model(cfg["model"], topo.device), meta, delta)
    if topo.rank == topo.leader:
        print(json.dumps(results, indent=2))
    topo.close()
    return results
