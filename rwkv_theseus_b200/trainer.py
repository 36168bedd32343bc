"""Parallel Layer Migration training loop (reference ``train.py:52-260``).

Per optimizer step and micro-batch: ONE frozen-teacher forward captures the
input (after ``input_layernorm``) and attention output of every full-attention
block; then, layer by layer, the TimeMix student of that block runs forward
and backward on the captured pair with its own carried state (detached at
chunk boundaries, reset at window boundaries). On the last micro-batch each
layer's gradient bucket is reduced across ranks and the layer is updated
(1/count scale, clip, AdamW) immediately, before the next layer's work.

Differences from the reference loop, all semantics-preserving:
* exhausted ranks contribute zero gradients and a zero token count to the
  explicit per-layer collective instead of running a dummy forward;
* count, grad norm and error flags stay on the device; the step's metrics are
  read with one device-to-host copy at the end of the step, where a
  non-finite norm or an empty update raises as ``clip_grad_norm_(...,
  error_if_nonfinite=True)`` / the token check would.
"""
import gc
import json
import os
import random
from pathlib import Path

import numpy as np
import torch

from .checkpoint import model_fingerprint, read_checkpoint, restore_rng, save_checkpoint, validate_resume, cpu_tree
from .config import steps_for
from .data import digest_file, reader_for
from .losses import metrics
from .models.hf_io import load_model
from .models.runner import Capture, Runner, install, migration_order, state_to_device
from .ops import native
from .parallel.topology import Topology
from .profiling import StepProfiler
from .schedule import lr_factor
from .stage import Student
from .tracking import Tracker
from .validation import summarize_layers, validate_composition, validate_parallel


def emit(topo, cfg, event, **fields):
    if topo.rank != topo.leader:
        return
    line = json.dumps({"event": event, **fields}, ensure_ascii=False)
    root = Path(cfg["output"])
    root.mkdir(parents=True, exist_ok=True)
    with (root / "metrics.jsonl").open("a") as f:
        f.write(line + "\n")
    if topo.tracker is not None:
        topo.tracker.log(event, fields)


def emit_profile(topo, cfg, step, phases):
    """``profile`` event: per-phase milliseconds of the step, maximum over ranks (Gloo gather)."""
    import torch.distributed as dist
    if topo.world > 1:
        everyone = [None] * topo.world
        dist.all_gather_object(everyone, phases)
    else:
        everyone = [phases]
    merged = {}
    for entry in everyone:
        for name, ms in entry.items():
            merged[name] = max(merged.get(name, 0.0), ms)
    teacher = merged.get("teacher", 0.0)
    students = sum(v for k, v in merged.items() if k.startswith("student_"))
    updates = sum(v for k, v in merged.items() if k.startswith("update_"))
    emit(topo, cfg, "profile", step=step, teacher_ms=teacher, students_ms=students, updates_ms=updates,
         exchange_join_ms=merged.get("exchange_join", 0.0), phases_ms=merged)


class StepEngine:
    """The hot loop body: teacher forward + per-layer student updates."""

    def __init__(self, cfg, topo, runner, order, students, captures):
        self.cfg, self.topo, self.runner = cfg, topo, runner
        self.order, self.students, self.captures = order, students, captures
        self.device = topo.device
        self._staging = [None, None]   # pinned id buffers, used alternately
        self._staged = [None, None]    # event after the copy out of each buffer
        self._turn = 0
        self.profiler = StepProfiler(self.device)
        if self.device.type == "cuda":
            for student in students.values():
                student.overlap_update = True

    def _to_device(self, ids):
        """Stage token ids through two persistent pinned buffers (alternating), copy asynchronously. A buffer
        is refilled only after the copy that last read it has run (its event), since the host may be more
        than a step ahead of the device."""
        if self.device.type != "cuda":
            return ids
        n, i = ids.numel(), self._turn
        self._turn ^= 1
        if self._staged[i] is not None:
            self._staged[i].synchronize()
        if self._staging[i] is None or self._staging[i].numel() < n:
            self._staging[i] = torch.empty(max(n, 1 << 16), dtype=torch.int64, pin_memory=True)
        host = self._staging[i][:n].view(ids.shape)
        host.copy_(ids)
        out = host.to(self.device, non_blocking=True)
        self._staged[i] = torch.cuda.Event()
        self._staged[i].record()
        return out

    def step(self, reader):
        """One optimizer update of every layer; returns per-layer device reports."""
        cfg, prof = self.cfg, self.profiler
        prof.reset()
        for micro in range(cfg["grad_accum_steps"]):
            batch = reader.next()
            if batch is not None:
                if batch["reset"]:
                    self.runner.reset()
                    for student in self.students.values():
                        student.state = None
                if self.runner.cache.cursor != batch["position"]:
                    raise RuntimeError("Cache position differs from consumed token stream")
                with prof.phase("teacher"):
                    self.runner.forward(self._to_device(batch["ids"]))
            last = micro == cfg["grad_accum_steps"] - 1
            for layer in self.order:
                student, capture = self.students[layer], self.captures[layer]
                if batch is not None:
                    with prof.phase(f"student_{layer:02d}"):
                        student.micro_step(capture.x, capture.y)
                    capture.x = capture.y = None
                if last:
                    with prof.phase(f"update_{layer:02d}"):
                        student.reduce()
                        student.update()
        with prof.phase("exchange_join"):
            self.topo.join_grad_sync()
        return {layer: s.report for layer, s in self.students.items()}

    def read_metrics(self, reports):
        """One device-to-host copy of all layer reports; raises on update errors."""
        for student in self.students.values():
            student.join_update()
        rows = torch.stack([reports[layer] for layer in self.order]).double().cpu().tolist()
        self.topo.check_grad_sync()
        if self.topo.device.type == "cuda" and native().gemm_fault():
            raise RuntimeError("a tcgen05 GEMM gave up a bounded wait (results of this step are invalid)")
        layer_metrics = {}
        for layer, (nmse, cos, count, norm, bad) in zip(self.order, rows):
            if count <= 0:
                raise RuntimeError("No training tokens in update")
            if bad or not np.isfinite(norm):
                raise RuntimeError(f"The total norm of gradients for layer {layer} is non-finite")
            student = self.students[layer]
            lr = self.cfg["lr"] * lr_factor(student.steps_done - 1, self.cfg, student.total_steps)
            layer_metrics[f"layer_{layer:02d}"] = metrics(torch.tensor([nmse, cos, count])) | {
                "grad_norm": norm, "lr": lr}
        return layer_metrics


def run(cfg, resume=None, stop_after=None):
    tracker = Tracker()
    try:
        _run(cfg, resume, stop_after, tracker)
    except BaseException:
        tracker.finish(exit_code=1)
        raise
    else:
        tracker.finish()


def _check_data(cfg):
    for manifest in (cfg["train_manifest"], cfg["validation_manifest"]):
        data = json.loads(Path(manifest).read_text())
        for source in data["sources"]:
            for field in ("tokens", "offsets"):
                if digest_file(Path(manifest).parent / source[field]) != source[field + "_sha256"]:
                    raise ValueError(f"Data content changed: {source[field]}")


def _check_vocab(cfg, model):
    for manifest in (cfg["train_manifest"], cfg["validation_manifest"]):
        data = json.loads(Path(manifest).read_text())
        if data["vocab_size"] > model.config.vocab_size:
            raise ValueError("Dataset vocabulary exceeds model embedding size")
        for name, expected in data.get("tokenizer_files", {}).items():
            token_file = Path(cfg["model"]) / name
            if not token_file.exists() or digest_file(token_file) != expected:
                raise ValueError(f"Dataset/model tokenizer differs: {name}")


def _run(cfg, resume, stop_after, tracker):
    from tqdm.auto import tqdm
    topo = Topology(cfg["distributed_backend"], cfg["timeout_minutes"])
    topo.tracker = tracker
    topo.assert_same({"config": cfg, "resume": resume, "stop_after": stop_after,
                      "profile": os.environ.get("THESEUS_PROFILE", "0")}, "run configuration")
    torch.set_num_threads(1)
    random.seed(cfg["seed"] + topo.rank)
    np.random.seed(cfg["seed"] + topo.rank)
    torch.manual_seed(cfg["seed"])
    if topo.rank == 0:
        _check_data(cfg)
    if not resume and (Path(cfg["output"]) / "latest").exists():
        raise ValueError("Output already has checkpoints; use --resume or a new output directory")
    topo.barrier()
    base_id = topo.broadcast_object(model_fingerprint(cfg["model"]) if topo.rank == topo.leader else None)
    model = load_model(cfg["model"], topo.device)
    _check_vocab(cfg, model)
    order = migration_order(model, cfg["expected_attention_layers"])
    if cfg["cosine_weight"] != 0:
        raise ValueError("Parallel migration requires cosine_weight=0")
    meta, delta, checkpoint = None, {}, None
    if resume:
        checkpoint, meta, delta = read_checkpoint(resume)
        if meta.get("training_topology") != "parallel_layers_v1":
            raise ValueError("Sequential checkpoints cannot resume parallel migration; start a new run")
        validate_resume(meta, cfg, topo, base_id, order)
        if set(delta) != set(order):
            raise ValueError("Checkpoint must contain every migration layer")
    export_meta = Path(cfg["output"]) / "converted" / "theseus.json"
    if meta and meta["complete"] and export_meta.exists():
        exported = json.loads(export_meta.read_text())
        if (exported.get("migration_fingerprint") != digest_file(checkpoint / "migrated.safetensors")
                or exported.get("base_fingerprint") != base_id):
            raise ValueError("Existing converted model differs from resumed checkpoint; choose a new output")
        topo.close()
        return
    saved = checkpoint
    tracker.start(cfg, topo, resume=bool(resume))
    runner = Runner(model)
    reader = reader_for(cfg, topo)
    if cfg["training_mode"] == "epoch":
        max_steps = (max(reader.rank_chunks) + cfg["grad_accum_steps"] - 1) // cfg["grad_accum_steps"]
    else:
        max_steps = steps_for(cfg, 0)
    step0 = meta["step"] if meta else 0
    students, captures = {}, {}
    for index, layer in enumerate(order):
        torch.manual_seed(cfg["seed"] + index)
        students[layer] = Student(model.config, layer, cfg, topo, delta.get(layer), total_steps=max_steps)
        captures[layer] = Capture(model.model.layers[layer].self_attn)
    if meta and not meta["complete"]:
        local = torch.load(checkpoint / "ranks" / f"rank_{topo.rank:05d}.pt", map_location="cpu", weights_only=False)
        runner.load_state_dict(local["runner"])
        reader.load_state_dict(local["reader"])
        opt = torch.load(checkpoint / "optimizer.pt", map_location=topo.device, weights_only=False)
        for layer, student in students.items():
            student.state = state_to_device(local["students"][layer], topo.device)
            student.load_optimizer_state(opt[layer]["optimizer"], opt[layer]["scheduler"])
            if student.steps_done != step0:
                raise ValueError("Checkpoint scheduler step differs from manifest step")
        restore_rng(local["rng"])
        del local, opt
    delta.clear()
    topo.barrier()
    engine = StepEngine(cfg, topo, runner, order, students, captures)
    progress = tqdm(total=max_steps, initial=step0, desc=f"Parallel migration ({len(order)} layers)",
                    unit="step", dynamic_ncols=True, mininterval=0.5,
                    disable=topo.rank != topo.leader or os.environ.get("TQDM_DISABLE") == "1")
    for step in range(step0 + 1, max_steps + 1):
        reports = engine.step(reader)
        layer_metrics = engine.read_metrics(reports)
        summary = summarize_layers(layer_metrics)
        progress.set_postfix(sum_loss=f"{summary['sum_loss']:.5f}", mean_cos=f"{summary['mean_cos']:.5f}",
                             refresh=False)
        progress.update(1)
        if step % cfg["log_interval"] == 0 or step == 1:
            emit(topo, cfg, "train", step=step, **summary,
                 tokens=next(iter(layer_metrics.values()))["tokens"], layers=layer_metrics)
        if engine.profiler.on:
            emit_profile(topo, cfg, step, engine.profiler.summary())
        complete = step == max_steps
        if complete and cfg["training_mode"] == "epoch" and not reader.exhausted:
            raise RuntimeError("Training ended before the local token shard was exhausted")
        if complete or (cfg["validation_interval"] and step % cfg["validation_interval"] == 0):
            result = validate_parallel(topo, cfg, runner, students, captures)
            emit(topo, cfg, "validation", step=step, **result)
        stopping = stop_after is not None and step - step0 >= stop_after
        if complete or stopping or (cfg["checkpoint_interval"] and step % cfg["checkpoint_interval"] == 0):
            saved = save_checkpoint(topo, cfg, step, complete, order, runner, reader, base_id, students)
            emit(topo, cfg, "checkpoint", path=str(saved), complete=complete)
        if stopping and not complete:
            progress.close()
            for capture in captures.values():
                capture.close()
            topo.close()
            return
    progress.close()
    for capture in captures.values():
        capture.close()
    topo.join_grad_sync()
    for s in students.values():
        s.sync_state()
    weights = {layer: cpu_tree(s.weights()) for layer, s in students.items()}
    students.clear()
    del runner, model, engine
    gc.collect()
    if topo.device.type == "cuda":
        torch.cuda.empty_cache()
    model = load_model(cfg["model"], topo.device)
    for layer in order:
        install(model, layer, cfg, weights[layer])
    del weights
    runner = Runner(model)
    result = validate_composition(topo, cfg, runner)
    emit(topo, cfg, "composition_validation", **result)
    if topo.rank == topo.leader:
        from .inference import save_export
        save_export(model, Path(cfg["output"]) / "converted", cfg, order, base_id, checkpoint=saved)
    topo.barrier()
    emit(topo, cfg, "finished", layers=len(order), export=str(Path(cfg["output"]) / "converted"))
    topo.close()
