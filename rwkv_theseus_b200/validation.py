"""Validation passes (reference ``theseus/validation.py:25-191``).

* ``validate_parallel``: every student scored teacher-forced at its own block
  (the teacher's captured input and attention output), on an isolated cache
  with temporary student states.
* ``validate_composition``: the assembled model (students in place of the
  attention blocks) runs the validation chunks; its output must be finite;
  optionally the KL against the original teacher.
* ``validate_original_kl``: the original attention blocks are rebuilt from the
  base safetensors for one isolated replay whose final hidden states (not
  logits) are kept; the assembled model's replay is then compared through
  ``lm_head`` in blocks of ``kl_token_block`` tokens.
* ``validate``: legacy single-stage validation of a sequential checkpoint
  (teacher-forced and free-running NMSE of one installed student).

Every pass reads the same ``validation_chunks`` chunks through ``replay``: an
isolated runner state, a cache reset at each window start, one teacher forward
per chunk, then the pass's own per-chunk work.
"""
from contextlib import contextmanager
from pathlib import Path

import torch
from safetensors import safe_open

from .data import reader_for
from .losses import kl_sum, metrics, statistics
from .models.hf_io import weight_map
from .models.qwen35 import Attention
from .models.runner import AttentionAdapter, Capture, isolated_state
from .models.timemix import detach_state


def summarize_layers(layers):
    """``sum_loss`` (sum of per-layer NMSE) and ``mean_cos`` over the layer metrics."""
    nmse = [entry["nmse"] for entry in layers.values()]
    cosine = [entry["cosine"] for entry in layers.values()]
    return {"sum_loss": sum(nmse), "mean_cos": sum(cosine) / len(cosine)}


def validation_batches(cfg, topo):
    """This rank's validation chunks (CPU batches), the same list for every pass."""
    reader = reader_for(cfg, topo, validation=True)
    return [reader.next() for _ in range(cfg["validation_chunks"])]


def replay(runner, batches, device, per_chunk, through_layer=None, on_reset=None):
    """Run `batches` through the teacher on an isolated state; ``per_chunk(index, output)`` after each forward,
    ``on_reset()`` whenever a new window starts."""
    with isolated_state(runner):
        for index, batch in enumerate(batches):
            if batch["reset"]:
                runner.reset()
                if on_reset is not None:
                    on_reset()
            out = runner.forward(batch["ids"].to(device), through_layer=through_layer)
            per_chunk(index, out)


def _layer_report(totals):
    layers = {f"layer_{layer:02d}": metrics(total) for layer, total in totals.items()}
    return summarize_layers(layers) | {"layers": layers}


@torch.no_grad()
def validate_parallel(topo, cfg, runner, students, captures):
    totals = {layer: torch.zeros(3, device=topo.device) for layer in students}
    states = dict.fromkeys(students)

    def forget():
        states.update(dict.fromkeys(students))

    def score(_, __):
        for layer, student in students.items():
            capture = captures[layer]
            prediction, states[layer] = student.predict(capture.x, states[layer])
            totals[layer] += statistics(prediction, capture.y, cfg["loss_epsilon"])
            capture.x = capture.y = None

    replay(runner, validation_batches(cfg, topo), topo.device, score, on_reset=forget)
    for total in totals.values():
        topo.student_sum(total)
    return _layer_report(totals)


def _original_block(model, layer, model_path, mapping, device):
    prefix = f"model.layers.{layer}.self_attn."
    names = {key: where for key, where in mapping.items() if key.startswith(prefix)}
    if not names:
        raise ValueError(f"Missing original attention {layer}")
    weights = {}
    for key, (shard, stored_as) in names.items():
        with safe_open(str(Path(model_path) / shard), framework="pt") as handle:
            weights[key[len(prefix):]] = handle.get_tensor(stored_as)
    block = Attention(model.config, layer)
    block.load_state_dict(weights, strict=True)
    return block.to(device=device, dtype=torch.bfloat16).requires_grad_(False).eval()


@contextmanager
def original_attention(model, model_path):
    """Within the block, every installed student is replaced by the base model's attention at its layer."""
    mapping = weight_map(Path(model_path))
    device = next(model.parameters()).device
    swapped = {}
    try:
        for layer, block in enumerate(model.model.layers):
            if isinstance(getattr(block, "self_attn", None), AttentionAdapter):
                swapped[layer] = block.self_attn
                block.self_attn = _original_block(model, layer, model_path, mapping, device)
        yield
    finally:
        for layer, adapter in swapped.items():
            model.model.layers[layer].self_attn = adapter


def _logits(hidden, head):
    """lm_head logits in the head's dtype (tcgen05 GEMM on CUDA bf16, matmul otherwise)."""
    if hidden.is_cuda and head.dtype == torch.bfloat16:
        from .ops.gemm import linear
        return linear(hidden.to(torch.bfloat16), head)
    return hidden.to(head.dtype) @ head.t()


@torch.no_grad()
def validate_original_kl(topo, cfg, runner):
    batches = validation_batches(cfg, topo)
    reference = [None] * len(batches)
    with original_attention(runner.model, cfg["model"]):
        replay(runner, batches, topo.device, lambda i, hidden: reference.__setitem__(i, hidden.cpu()))
    total = torch.zeros(2, device=topo.device)
    head = runner.model.lm_head.weight
    block = cfg["kl_token_block"]

    def compare(index, hidden):
        teacher = reference[index]
        for start in range(0, hidden.shape[1], block):
            student_logits = _logits(hidden[:, start:start + block], head)
            teacher_logits = _logits(teacher[:, start:start + block].to(topo.device), head)
            total[0] += kl_sum(student_logits, teacher_logits)
            total[1] += student_logits.shape[0] * student_logits.shape[1]

    replay(runner, batches, topo.device, compare)
    topo.student_sum(total)
    return {"original_teacher_kl": (total[0] / total[1]).item()}


@torch.no_grad()
def validate_composition(topo, cfg, runner):
    def finite(_, hidden):
        if not torch.isfinite(hidden).all():
            raise RuntimeError("Nonfinite assembled model output")

    replay(runner, validation_batches(cfg, topo), topo.device, finite)
    report = {"finite": True}
    if cfg["original_teacher_kl"]:
        report |= validate_original_kl(topo, cfg, runner)
    return report


@torch.no_grad()
def validate(topo, cfg, runner, layer):
    """Legacy sequential-stage validation of the student installed at `layer`: its teacher-forced NMSE (fed the
    teacher's own block input) and its free-running NMSE inside the assembled forward, against the teacher's
    attention output at that block."""
    adapter = runner.model.model.layers[layer].self_attn
    batches = validation_batches(cfg, topo)
    topo.barrier()
    targets = []
    watch = Capture(adapter.teacher)
    adapter.teacher_mode = True
    try:
        replay(runner, batches, topo.device, lambda *_: targets.append((watch.x.cpu(), watch.y.cpu())),
               through_layer=layer)
    finally:
        adapter.teacher_mode = False
        watch.close()
    sums = torch.zeros((2, 3), device=topo.device)   # [teacher-forced, free-running] x [nmse, cos, count]
    forced = {"state": None}
    watch = Capture(adapter)

    def score(index, _):
        x, y = (t.to(topo.device) for t in targets[index])
        sums[1] += statistics(watch.y, y, cfg["loss_epsilon"])
        with torch.autocast(topo.device.type, dtype=torch.bfloat16):
            prediction, state = adapter.core(x, forced["state"])
        forced["state"] = detach_state(state)
        sums[0] += statistics(prediction, y, cfg["loss_epsilon"])

    try:
        replay(runner, batches, topo.device, score, on_reset=lambda: forced.update(state=None))
    finally:
        watch.close()
    topo.student_sum(sums)
    report = {"teacher_forced": metrics(sums[0]), "student_forward": metrics(sums[1])}
    if cfg["original_teacher_kl"]:
        report |= validate_original_kl(topo, cfg, runner)
    topo.barrier()
    return report
