"""Parallel Layer Migration training (reference ``train.py:52-260``).

Per optimizer step and micro-batch: ONE frozen-teacher forward captures, at
every full-attention block, the attention input (after ``input_layernorm``)
and output; then, layer by layer, that block's TimeMix student runs forward and
backward on the captured pair with its own carried state (detached between
chunks, reset at window starts). On the last micro-batch each layer's gradients
are reduced across ranks and the layer is updated (1/count, clip, AdamW) right
away, before the next layer's work.

Semantics kept from the reference, mechanics of this implementation:
* exhausted ranks add zero gradients and a zero token count to the explicit
  per-layer reduction instead of running a dummy forward;
* the teacher forward ends at the last migrated block's attention output (the
  blocks after it, its MLP and the final norm feed no capture);
* token count, grad norm and error flags stay on the device; one asynchronous copy
  per step brings them to the host, which reads step s while step s + 1 runs and
  raises there, as ``clip_grad_norm_(..., error_if_nonfinite=True)`` and the token
  check would (before any validation, checkpoint or stop the step is read first);
* with the peer-memory exchange each layer's update runs on a side stream and
  the layer's next use waits for it (no step-wide join).

``MigrationJob`` is the whole run (set-up, resume, steps with logging,
validation and checkpoints, final assembly and export); ``StepEngine`` is the
hot loop body that ``bench.py`` also drives.
"""
import gc
import json
import os
import random
from contextlib import nullcontext
from pathlib import Path

import numpy as np
import torch

from .checkpoint import cpu_tree, model_fingerprint, read_checkpoint, restore_rng, save_checkpoint, validate_resume
from .config import steps_for
from .data import sha256_of_file, reader_for
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


class Journal:
    """``metrics.jsonl`` in the output directory plus the tracker; written by the leader only."""

    def __init__(self, topo, cfg):
        self.topo = topo
        self.path = Path(cfg["output"]) / "metrics.jsonl"

    def __call__(self, event, **fields):
        if self.topo.rank != self.topo.leader:
            return
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with self.path.open("a") as sink:
            sink.write(json.dumps({"event": event, **fields}, ensure_ascii=False) + "\n")
        if self.topo.tracker is not None:
            self.topo.tracker.log(event, fields)


def emit(topo, cfg, event, **fields):
    Journal(topo, cfg)(event, **fields)


def emit_profile(topo, cfg, step, phases):
    """``profile`` event: per-phase milliseconds of the step, maximum over ranks (Gloo gather)."""
    import torch.distributed as dist
    per_rank = [phases]
    if topo.world > 1:
        per_rank = [None] * topo.world
        dist.all_gather_object(per_rank, phases)
    slowest = {}
    for entry in per_rank:
        for name, ms in entry.items():
            slowest[name] = max(slowest.get(name, 0.0), ms)
    by_kind = lambda prefix: sum(ms for name, ms in slowest.items() if name.startswith(prefix))  # noqa: E731
    emit(topo, cfg, "profile", step=step, teacher_ms=slowest.get("teacher", 0.0), students_ms=by_kind("student_"),
         updates_ms=by_kind("update_"), exchange_join_ms=slowest.get("exchange_join", 0.0), phases_ms=slowest)


class StepEngine:
    """One optimizer step of every layer: teacher forward(s), per-layer micro-steps and updates."""

    def __init__(self, cfg, topo, runner, order, students, captures):
        self.cfg, self.topo, self.runner = cfg, topo, runner
        self.order, self.students, self.captures = order, students, captures
        self.device = topo.device
        self.last_capture = max(order)
        self.profiler = StepProfiler(self.device)
        # [layers, 5] the step's reports: each student's report is a row of this tensor (written in place by its
        # update on the update stream), so the whole step's reports leave in one copy
        self._snap = torch.zeros(len(order), 5, device=self.device)
        for index, layer in enumerate(order):
            students[layer].report = self._snap[index]
        self._slot = 0                        # pinned metric buffers used in turn
        self._pinned_rows = [None, None]
        self._pinned_faults = [None, None]
        self._pinned_status = [None, None]
        self._pending_events = [(), ()]
        self._pinned = [None, None]   # two pinned id buffers used in turn
        self._copied = [None, None]   # event after the copy that last read each buffer
        self._turn = 0
        # On CUDA a step's per-layer updates (local AdamW, or the peer exchange) are issued at the start of the next
        # step, on their side stream, so that they run under its teacher forward (which reads no student parameter)
        # instead of competing with the next layers' student work; each layer's next micro-step waits for its own.
        self.defer_updates = self.device.type == "cuda"
        self._deferred = []           # students whose update of the last step is not issued yet
        self._waiting_reads = []      # metric reads of that step, issued right after its updates
        if self.device.type == "cuda":
            for student in students.values():
                student.overlap_update = True
        # On CUDA (config ``overlap_students``) the micro-steps run on a stream of their own: student L waits only
        # for the event its capture records after layer L's attention, so it runs beside the rest of the teacher
        # forward and fills the SMs that the teacher's latency-bound kernels (GDN state pass, attention tail) leave
        # idle. Its GEMMs use the second stream-K workspace (lane 1); parallel split-K runs as stream-K while two
        # lanes can overlap. Nothing joins the streams at the end of a step: the next step's teacher forward starts
        # beside the last students; the deferred updates and the metric copies are issued on the student stream,
        # and ``join_students`` / ``join_updates`` order later reads after the students.
        self.student_stream = None
        self._compute = None
        if self.device.type == "cuda" and cfg.get("overlap_students", True):
            # THESEUS_STUDENT_PRIORITY: CUDA priority of the student stream (0, the default, is the lowest and the
            # compute stream's; -1 makes the block scheduler prefer student kernels when both streams have work).
            priority = int(os.environ.get("THESEUS_STUDENT_PRIORITY", "0"))
            self.student_stream = torch.cuda.Stream(self.device, priority=priority)
            native().gemm_set_concurrent(True)
            for capture in captures.values():
                capture.record_events = True

    def _to_device(self, ids):
        """Token ids to the device through two alternating pinned buffers (asynchronous copy). A buffer is
        refilled only after the copy that last read it ran, since the host may run ahead of the device."""
        if self.device.type != "cuda":
            return ids
        slot = self._turn
        self._turn ^= 1
        if self._copied[slot] is not None:
            self._copied[slot].synchronize()
        if self._pinned[slot] is None or self._pinned[slot].numel() < ids.numel():
            self._pinned[slot] = torch.empty(max(ids.numel(), 1 << 16), dtype=torch.int64, pin_memory=True)
        staged = self._pinned[slot][:ids.numel()].view(ids.shape)
        staged.copy_(ids)
        on_device = staged.to(self.device, non_blocking=True)
        self._copied[slot] = torch.cuda.Event()
        self._copied[slot].record()
        return on_device

    def _teacher(self, batch):
        if batch["reset"]:
            self.runner.reset()
            for student in self.students.values():
                student.state = None
        if self.runner.cache.cursor != batch["position"]:
            raise RuntimeError("Cache position differs from consumed token stream")
        with self.profiler.phase("teacher"):
            self.runner.forward(self._to_device(batch["ids"]), through_layer=self.last_capture)

    def step(self, reader):
        """One optimizer update of every layer; returns {layer: device report [nmse, cos, count, norm, error]}.
        The reports are rows of one engine tensor, written on the stream their updates ran on, so that
        ``read_metrics_async`` can read a step while the next one already runs."""
        profiler = self.profiler
        profiler.reset()
        if self.device.type == "cuda":
            self._compute = torch.cuda.current_stream(self.device)  # the teacher's stream
        self.flush()  # the previous step's updates, under this step's teacher forward
        micro_steps = self.cfg["grad_accum_steps"]
        for micro in range(micro_steps):
            batch = reader.next()
            if batch is not None:
                self._teacher(batch)
            updating = micro == micro_steps - 1
            for layer in self.order:
                student, capture = self.students[layer], self.captures[layer]
                if batch is not None:
                    self._micro_step(student, capture, f"student_{layer:02d}")
                    capture.x = capture.y = None
                if updating:
                    if self.defer_updates:
                        self._deferred.append(student)
                    else:  # right after the micro-step, on the stream it ran on
                        with self._on_student_stream(), profiler.phase(f"update_{layer:02d}"):
                            student.reduce()
                            student.update()
        return {layer: student.report for layer, student in self.students.items()}

    def join_students(self):
        """Make the current stream wait for every student micro-step issued so far (the step itself does not: the
        next step's teacher forward starts while the last students of this one still run)."""
        if self.student_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.student_stream)

    def _on_student_stream(self):
        return torch.cuda.stream(self.student_stream) if self.student_stream is not None else nullcontext()

    def _micro_step(self, student, capture, phase):
        stream = self.student_stream
        if stream is None or capture.ready is None:
            with self.profiler.phase(phase):
                student.micro_step(capture.x, capture.y)
            return
        x, y = capture.x, capture.y
        stream.wait_event(capture.ready)
        carried = () if student.state is None else tuple(student.state.values())
        for tensor in (x, y, *carried):  # allocated on other streams: not reused before the student stream is done
            tensor.record_stream(stream)
        ext = native()
        with torch.cuda.stream(stream), self.profiler.phase(phase):
            ext.gemm_set_lane(1)
            try:
                student.micro_step(x, y)
            finally:
                ext.gemm_set_lane(0)
        capture.ready = None

    def join_updates(self):
        """Issue any deferred updates and make the current stream wait for every layer's update (local AdamW or
        peer exchange): after this, work recorded on the current stream follows all of them."""
        self.flush()
        self.join_students()
        for student in self.students.values():
            student.join_update()

    def flush(self):
        """Issue the updates deferred from the last step (in layer order, the same on every rank) and the metric
        reads waiting for them. Called at the start of every step; call it before anything that reads student
        parameters outside a step (validation, checkpoints, export) or before a step-exact device timing ends."""
        deferred, self._deferred = self._deferred, []
        waiting, self._waiting_reads = self._waiting_reads, []
        with self._on_student_stream():  # the updates and metric copies follow the students' last micro-steps
            for student in deferred:
                with self.profiler.phase(f"update_{student.layer:02d}"):
                    student.reduce()
                    student.update()
            for pending in waiting:
                self._issue_read(pending)

    # ---------------------------------------------------------------- metrics

    def read_metrics_async(self, reports):
        """Start bringing this step's reports, the kernels' fault words and the exchange status to the host; returns
        a ``PendingMetrics`` whose ``result()`` waits for them and validates. The host may issue the next step in
        between. The reports and the exchange status are copied on the stream the updates ran on (ordered after
        this step's updates and before the next step's); the fault words are copied and cleared on the current
        stream, in order with the kernels that set them. With deferred updates the copies are issued right after
        the updates, at the start of the next step (or by ``flush``, which ``result()`` calls if needed)."""
        if self.device.type != "cuda":
            pending = PendingMetrics(self)
            lrs = self._learning_rates()
            pending.issued(torch.stack([reports[layer] for layer in self.order]), None, None, (), lrs)
            return pending
        pending = PendingMetrics(self)
        if self._deferred:
            self._waiting_reads.append(pending)
        else:
            self._issue_read(pending)
        return pending

    def _learning_rates(self):
        """Learning rate each layer's last update used."""
        return [self.cfg["lr"] * lr_factor(self.students[layer].steps_done - 1, self.cfg,
                                           self.students[layer].total_steps) for layer in self.order]

    def _issue_read(self, pending):
        slot = self._slot
        self._slot ^= 1
        for event in self._pending_events[slot]:
            event.synchronize()  # the host has read that slot's previous step
        if self._pinned_rows[slot] is None:
            self._pinned_rows[slot] = torch.empty(len(self.order), 5, pin_memory=True)
            self._pinned_faults[slot] = torch.zeros(3, dtype=torch.int32, pin_memory=True)
            self._pinned_status[slot] = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        first = self.students[self.order[0]]
        exchange = first._exchange()
        main = torch.cuda.current_stream(self.device)
        side = first.update_stream() or main
        with torch.cuda.stream(side):
            self._pinned_rows[slot].copy_(self._snap, non_blocking=True)
            if exchange is not None:
                self._pinned_status[slot].copy_(exchange.status_words(), non_blocking=True)
            reports_copied = torch.cuda.Event()
            reports_copied.record(side)
        if self.student_stream is not None:  # after the students' kernels and the teacher's (which precede them)
            self.student_stream.wait_stream(self._compute or main)
            main = self.student_stream
        with torch.cuda.stream(main):
            native().fault_words_async(self._pinned_faults[slot])
        faults_copied = torch.cuda.Event()
        faults_copied.record(main)
        self._pending_events[slot] = (reports_copied, faults_copied)
        pending.issued(self._pinned_rows[slot], self._pinned_faults[slot],
                       self._pinned_status[slot] if exchange is not None else None, self._pending_events[slot],
                       self._learning_rates())

    def read_metrics(self, reports):
        """Synchronous form: the validated metrics of the step that produced `reports`."""
        return self.read_metrics_async(reports).result()

    def _validate(self, rows, faults, status, lrs):
        if status is not None:
            self.topo.grad_sync().raise_for(status)
        if faults is not None and faults[0]:
            native().gemm_fault()  # resets the GEMM schedule counters before the error propagates
            raise RuntimeError("a tcgen05 GEMM gave up a bounded wait (results of this step are invalid)")
        if faults is not None and (faults[1] or faults[2]):
            raise RuntimeError(f"a tcgen05 WKV7 kernel gave up a bounded wait (fault words {faults[1]:#x}, "
                               f"{faults[2]:#x}; results of this step are invalid)")
        report = {}
        for layer, (nmse, cos, count, norm, bad), lr in zip(self.order, rows, lrs):
            if count <= 0:
                raise RuntimeError("No training tokens in update")
            if bad or not np.isfinite(norm):
                raise RuntimeError(f"The total norm of gradients for layer {layer} is non-finite")
            report[f"layer_{layer:02d}"] = metrics(torch.tensor([nmse, cos, count])) | {"grad_norm": norm, "lr": lr}
        return report


class PendingMetrics:
    """One step's metrics on their way to the host (``StepEngine.read_metrics_async``)."""

    def __init__(self, engine):
        self.engine = engine
        self.rows = None  # set when the copies are issued
        self._value = None

    def issued(self, rows, faults, status, events, lrs):
        self.rows, self.faults, self.status, self.events, self.lrs = rows, faults, status, events, lrs

    def result(self):
        if self._value is None:
            if self.rows is None:
                self.engine.flush()  # the step's updates (and with them this read) were still deferred
            for event in self.events:
                event.synchronize()
            rows = self.rows.double().tolist()
            faults = None if self.faults is None else self.faults.tolist()
            status = None if self.status is None else self.status.tolist()
            self._value = self.engine._validate(rows, faults, status, self.lrs)
        return self._value


def run(cfg, resume=None, stop_after=None):
    """Train (or resume) a migration run end to end; the tracker is closed with the run's outcome."""
    tracker = Tracker()
    try:
        MigrationJob(cfg, resume, stop_after, tracker).run()
    except BaseException:
        tracker.finish(exit_code=1)
        raise
    tracker.finish()


class MigrationJob:
    def __init__(self, cfg, resume, stop_after, tracker):
        self.cfg, self.resume, self.stop_after, self.tracker = cfg, resume, stop_after, tracker
        self.checkpoint = self.meta = None
        self.delta = {}

    # ---------------------------------------------------------------- set-up
    def _agree_and_seed(self):
        topo, cfg = self.topo, self.cfg
        topo.assert_same({"config": cfg, "resume": self.resume, "stop_after": self.stop_after,
                          "profile": os.environ.get("THESEUS_PROFILE", "0")}, "run configuration")
        torch.set_num_threads(1)
        random.seed(cfg["seed"] + topo.rank)
        np.random.seed(cfg["seed"] + topo.rank)
        torch.manual_seed(cfg["seed"])

    def _manifests(self):
        return [(manifest, json.loads(Path(manifest).read_text()))
                for manifest in (self.cfg["train_manifest"], self.cfg["validation_manifest"])]

    def _check_data_bytes(self):
        for manifest, spec in self._manifests():
            for source in spec["sources"]:
                for field in ("tokens", "offsets"):
                    if sha256_of_file(Path(manifest).parent / source[field]) != source[f"{field}_sha256"]:
                        raise ValueError(f"Data content changed: {source[field]}")

    def _check_data_fits_model(self):
        for _, spec in self._manifests():
            if spec["vocab_size"] > self.model.config.vocab_size:
                raise ValueError("Dataset vocabulary exceeds model embedding size")
            for name, expected in spec.get("tokenizer_files", {}).items():
                found = Path(self.cfg["model"]) / name
                if not found.exists() or sha256_of_file(found) != expected:
                    raise ValueError(f"Dataset/model tokenizer differs: {name}")

    def _open(self):
        cfg = self.cfg
        self.topo = Topology(cfg["distributed_backend"], cfg["timeout_minutes"])
        self.topo.tracker = self.tracker
        self.journal = Journal(self.topo, cfg)
        self._agree_and_seed()
        if self.topo.rank == 0:
            self._check_data_bytes()   # before any model allocation
        if not self.resume and (Path(cfg["output"]) / "latest").exists():
            raise ValueError("Output already has checkpoints; use --resume or a new output directory")
        self.topo.barrier()
        leader = self.topo.rank == self.topo.leader
        self.base_id = self.topo.broadcast_object(model_fingerprint(cfg["model"]) if leader else None)
        self.model = load_model(cfg["model"], self.topo.device)
        self._check_data_fits_model()
        self.order = migration_order(self.model, cfg["expected_attention_layers"])
        if cfg["cosine_weight"] != 0:
            raise ValueError("Parallel migration requires cosine_weight=0")

    def _load_resume(self):
        """Read the checkpoint to resume. True when it is complete and already exported (nothing left to do)."""
        if not self.resume:
            return False
        self.checkpoint, self.meta, self.delta = read_checkpoint(self.resume)
        if self.meta.get("training_topology") != "parallel_layers_v1":
            raise ValueError("Sequential checkpoints cannot resume parallel migration; start a new run")
        validate_resume(self.meta, self.cfg, self.topo, self.base_id, self.order)
        if set(self.delta) != set(self.order):
            raise ValueError("Checkpoint must contain every migration layer")
        exported = Path(self.cfg["output"]) / "converted" / "theseus.json"
        if not (self.meta["complete"] and exported.exists()):
            return False
        record = json.loads(exported.read_text())
        if (record.get("migration_fingerprint") != sha256_of_file(self.checkpoint / "migrated.safetensors")
                or record.get("base_fingerprint") != self.base_id):
            raise ValueError("Existing converted model differs from resumed checkpoint; choose a new output")
        return True

    def _build(self):
        cfg = self.cfg
        self.runner = Runner(self.model)
        self.reader = reader_for(cfg, self.topo)
        if cfg["training_mode"] == "epoch":
            self.max_steps = -(-max(self.reader.rank_chunks) // cfg["grad_accum_steps"])
        else:
            self.max_steps = steps_for(cfg, 0)
        self.step0 = self.meta["step"] if self.meta else 0
        self.students, self.captures = {}, {}
        for index, layer in enumerate(self.order):
            torch.manual_seed(cfg["seed"] + index)  # the same per-layer init stream as the reference
            self.students[layer] = Student(self.model.config, layer, cfg, self.topo, self.delta.get(layer),
                                           total_steps=self.max_steps)
            self.captures[layer] = Capture(self.model.model.layers[layer].self_attn)
        if self.meta and not self.meta["complete"]:
            self._restore_midstream()
        self.delta = {}
        self.topo.barrier()
        self.engine = StepEngine(cfg, self.topo, self.runner, self.order, self.students, self.captures)

    def _restore_midstream(self):
        device = self.topo.device
        mine = torch.load(self.checkpoint / "ranks" / f"rank_{self.topo.rank:05d}.pt", map_location="cpu",
                          weights_only=False)
        self.runner.load_state_dict(mine["runner"])
        self.reader.load_state_dict(mine["reader"])
        optimizer = torch.load(self.checkpoint / "optimizer.pt", map_location=device, weights_only=False)
        for layer, student in self.students.items():
            student.state = state_to_device(mine["students"][layer], device)
            student.load_optimizer_state(optimizer[layer]["optimizer"], optimizer[layer]["scheduler"])
            if student.steps_done != self.step0:
                raise ValueError("Checkpoint scheduler step differs from manifest step")
        restore_rng(mine["rng"])

    # ---------------------------------------------------------------- steps
    def _log_step(self, step, layer_metrics, progress):
        summary = summarize_layers(layer_metrics)
        progress.set_postfix(sum_loss=f"{summary['sum_loss']:.5f}", mean_cos=f"{summary['mean_cos']:.5f}",
                             refresh=False)
        progress.update(1)
        if step == 1 or step % self.cfg["log_interval"] == 0:
            tokens = next(iter(layer_metrics.values()))["tokens"]
            self.journal("train", step=step, **summary, tokens=tokens, layers=layer_metrics)
        if self.engine.profiler.on:
            emit_profile(self.topo, self.cfg, step, self.engine.profiler.summary())

    def _due(self, step, interval_key, complete):
        interval = self.cfg[interval_key]
        return complete or bool(interval and step % interval == 0)

    def _train(self):
        """The step loop. Returns False when ``stop_after`` ended it before the last step."""
        from tqdm.auto import tqdm
        cfg = self.cfg
        progress = tqdm(total=self.max_steps, initial=self.step0, unit="step", dynamic_ncols=True,
                        desc=f"Parallel migration ({len(self.order)} layers)", mininterval=0.5,
                        disable=self.topo.rank != self.topo.leader or os.environ.get("TQDM_DISABLE") == "1")
        self.saved = self.checkpoint
        pending = None  # (step, PendingMetrics) read after the next step is issued
        try:
            for step in range(self.step0 + 1, self.max_steps + 1):
                reports = self.engine.step(self.reader)
                if pending is not None:
                    self._log_step(pending[0], pending[1].result(), progress)
                pending = (step, self.engine.read_metrics_async(reports))
                complete = step == self.max_steps
                stopping = self.stop_after is not None and step - self.step0 >= self.stop_after
                boundary = (complete or stopping or self.engine.profiler.on
                            or self._due(step, "validation_interval", complete)
                            or self._due(step, "checkpoint_interval", complete))
                if boundary:  # validation, checkpoint, stop and profiling act on a finished, logged step
                    self._log_step(pending[0], pending[1].result(), progress)
                    pending = None
                if complete and cfg["training_mode"] == "epoch" and not self.reader.exhausted:
                    raise RuntimeError("Training ended before the local token shard was exhausted")
                if self._due(step, "validation_interval", complete):
                    result = validate_parallel(self.topo, cfg, self.runner, self.students, self.captures)
                    self.journal("validation", step=step, **result)
                if stopping or self._due(step, "checkpoint_interval", complete):
                    self.saved = save_checkpoint(self.topo, cfg, step, complete, self.order, self.runner,
                                                 self.reader, self.base_id, self.students)
                    self.journal("checkpoint", path=str(self.saved), complete=complete)
                if stopping and not complete:
                    return False
            if pending is not None:
                self._log_step(pending[0], pending[1].result(), progress)
            return True
        finally:
            progress.close()
            for capture in self.captures.values():
                capture.close()

    # ---------------------------------------------------------------- assembly
    def _assemble_and_export(self):
        """Reload the pristine base, install every trained student in place of its attention, validate the
        assembled model and write the export."""
        cfg = self.cfg
        self.topo.join_grad_sync()
        for student in self.students.values():
            student.sync_state()
        trained = {layer: cpu_tree(student.weights()) for layer, student in self.students.items()}
        self.students.clear()
        self.runner = self.model = self.engine = None
        gc.collect()
        if self.topo.device.type == "cuda":
            torch.cuda.empty_cache()
        self.model = load_model(cfg["model"], self.topo.device)
        for layer in self.order:
            install(self.model, layer, cfg, trained.pop(layer))
        result = validate_composition(self.topo, cfg, Runner(self.model))
        self.journal("composition_validation", **result)
        export = Path(cfg["output"]) / "converted"
        if self.topo.rank == self.topo.leader:
            from .inference import save_export
            save_export(self.model, export, cfg, self.order, self.base_id, checkpoint=self.saved)
        self.topo.barrier()
        self.journal("finished", layers=len(self.order), export=str(export))

    def run(self):
        self._open()
        if self._load_resume():
            self.topo.close()
            return
        self.tracker.start(self.cfg, self.topo, resume=bool(self.resume))
        self._build()
        if self._train():
            self._assemble_and_export()
        self.topo.close()
