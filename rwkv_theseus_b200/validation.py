"""Validation passes (reference ``theseus/validation.py:25-191``).

* ``validate_parallel``: every student scored teacher-forced on the teacher's
  own boundaries, with an isolated cache and temporary student states.
* ``validate_composition``: the assembled model (students installed in place
  of attention) runs the validation chunks; output must be finite; optional
  KL against the original teacher.
* ``validate_original_kl``: rebuilds each original attention block from the
  base safetensors for one isolated replay, stores hidden states (not logits)
  and compares ``lm_head`` distributions in blocks of ``kl_token_block``.
* ``validate``: legacy single-stage validation of a sequential checkpoint.
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
    return {"sum_loss": sum(item["nmse"] for item in layers.values()),
            "mean_cos": sum(item["cosine"] for item in layers.values()) / len(layers)}


@torch.no_grad()
def validate_parallel(topo, cfg, runner, students, captures):
    totals = {i: torch.zeros(3, device=topo.device) for i in students}
    states = {i: None for i in students}
    reader = reader_for(cfg, topo, validation=True)
    with isolated_state(runner):
        for _ in range(cfg["validation_chunks"]):
            batch = reader.next()
            if batch["reset"]:
                runner.reset()
                states = {i: None for i in students}
            runner.forward(batch["ids"].to(topo.device))
            for i, student in students.items():
                capture = captures[i]
                prediction, states[i] = student.predict(capture.x, states[i])
                totals[i] += statistics(prediction, capture.y, cfg["loss_epsilon"])
                capture.x = capture.y = None
    for total in totals.values():
        topo.student_sum(total)
    layers = {f"layer_{i:02d}": metrics(total) for i, total in totals.items()}
    return summarize_layers(layers) | {"layers": layers}


@contextmanager
def original_attention(model, model_path):
    """Temporarily restore the base model's attention blocks in place of students."""
    path = Path(model_path)
    mapping = weight_map(path)
    device = next(model.parameters()).device
    originals = {}
    try:
        for i, block in enumerate(model.model.layers):
            current = getattr(block, "self_attn", None)
            if not isinstance(current, AttentionAdapter):
                continue
            originals[i] = current
            prefix = f"model.layers.{i}.self_attn."
            keys = {k: v for k, v in mapping.items() if k.startswith(prefix)}
            if not keys:
                raise ValueError(f"Missing original attention {i}")
            module = Attention(model.config, i)
            state = {}
            for name, (shard, raw) in keys.items():
                with safe_open(str(path / shard), framework="pt") as f:
                    state[name[len(prefix):]] = f.get_tensor(raw)
            module.load_state_dict(state, strict=True)
            block.self_attn = module.to(device=device, dtype=torch.bfloat16).requires_grad_(False).eval()
        yield
    finally:
        for i, module in originals.items():
            model.model.layers[i].self_attn = module


@torch.no_grad()
def validate_original_kl(topo, cfg, runner):
    reader = reader_for(cfg, topo, validation=True)
    batches = [reader.next() for _ in range(cfg["validation_chunks"])]
    teacher_hidden = []
    with isolated_state(runner):
        with original_attention(runner.model, cfg["model"]):
            runner.reset()
            for batch in batches:
                if batch["reset"]:
                    runner.reset()
                teacher_hidden.append(runner.forward(batch["ids"].to(topo.device)).cpu())
    total = torch.zeros(2, device=topo.device)
    head = runner.model.lm_head.weight
    with isolated_state(runner):
        for batch, teacher in zip(batches, teacher_hidden):
            if batch["reset"]:
                runner.reset()
            hidden = runner.forward(batch["ids"].to(topo.device))
            for start in range(0, hidden.shape[1], cfg["kl_token_block"]):
                stop = start + cfg["kl_token_block"]
                logits = _logits(hidden[:, start:stop], head)
                target = _logits(teacher[:, start:stop].to(topo.device), head)
                total[0] += kl_sum(logits, target)
                total[1] += logits.shape[0] * logits.shape[1]
    topo.student_sum(total)
    return {"original_teacher_kl": (total[0] / total[1]).item()}


def _logits(hidden, head):
    """lm_head logits in the head's dtype (tcgen05 GEMM on CUDA bf16, matmul otherwise)."""
    if hidden.is_cuda and head.dtype == torch.bfloat16:
        from .ops.gemm import linear
        return linear(hidden.to(torch.bfloat16), head)
    return hidden.to(head.dtype) @ head.t()


@torch.no_grad()
def validate_composition(topo, cfg, runner):
    reader = reader_for(cfg, topo, validation=True)
    with isolated_state(runner):
        for _ in range(cfg["validation_chunks"]):
            batch = reader.next()
            if batch["reset"]:
                runner.reset()
            hidden = runner.forward(batch["ids"].to(topo.device))
            if not torch.isfinite(hidden).all():
                raise RuntimeError("Nonfinite assembled model output")
    results = {"finite": True}
    if cfg["original_teacher_kl"]:
        results.update(validate_original_kl(topo, cfg, runner))
    return results


@torch.no_grad()
def validate(topo, cfg, runner, layer):
    """Legacy sequential-stage validation: teacher-forced and free-running NMSE of one layer."""
    adapter = runner.model.model.layers[layer].self_attn
    total = torch.zeros((2, 3), device=topo.device)
    reader = reader_for(cfg, topo, validation=True)
    batches = [reader.next() for _ in range(cfg["validation_chunks"])]
    targets = []
    topo.barrier()
    with isolated_state(runner):
        capture = Capture(adapter.teacher)
        adapter.teacher_mode = True
        try:
            for batch in batches:
                if batch["reset"]:
                    runner.reset()
                runner.forward(batch["ids"].to(topo.device), through_layer=layer)
                targets.append((capture.x.cpu(), capture.y.cpu()))
        finally:
            adapter.teacher_mode = False
            capture.close()
    with isolated_state(runner):
        capture = Capture(adapter)
        forced_state = None
        try:
            for batch, (x, y) in zip(batches, targets):
                if batch["reset"]:
                    runner.reset()
                    forced_state = None
                x, y = x.to(topo.device), y.to(topo.device)
                runner.forward(batch["ids"].to(topo.device))
                total[1] += statistics(capture.y, y, cfg["loss_epsilon"])
                with torch.autocast(topo.device.type, dtype=torch.bfloat16):
                    forced, forced_state = adapter.core(x, forced_state)
                forced_state = detach_state(forced_state)
                total[0] += statistics(forced, y, cfg["loss_epsilon"])
        finally:
            capture.close()
    topo.student_sum(total)
    results = {"teacher_forced": metrics(total[0]), "student_forward": metrics(total[1])}
    if cfg["original_teacher_kl"]:
        results.update(validate_original_kl(topo, cfg, runner))
    topo.barrier()
    return results
