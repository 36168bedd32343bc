#!/usr/bin/env python3
"""Headline benchmark: Parallel Layer Migration training tokens/s on the 27B hybrid.

Config: Qwen3.5-style hybrid teacher, bf16, random init
(vocab 248077, hidden 5120, 64 blocks, every 4th full attention with 24/4
heads x 256, GDN 16/48 heads x 128, conv 4, SwiGLU 17408) and sixteen RWKV7
TimeMix students (head size 64) trained with AdamW; synthetic documents with
log-uniform lengths in [256, 16384] and uniform token ids; context 4096,
chunk 1024, micro-batch 1; one process per GPU, each rank on its own data
shard (weak scaling).

A step is one optimizer update of all sixteen layers on one chunk: one
teacher forward, sixteen student forward/backward passes, sixteen gradient
reductions (world > 1) and sixteen clip+AdamW updates. The engine issues a
step's updates at the start of the next step (they run under its teacher
forward); the timed region starts after the warm-up's updates completed and
its end event waits for the K-th step's updates (side streams included), so
it holds exactly K steps of work.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
device synchronisation, timed with CUDA events; the reported number is the
total token count over all ranks divided by the slowest rank's time. The
working set (54 GB of teacher weights per step) exceeds L2, so no flush is
needed between steps. ``e2e`` runs the same K batches again (reader, teacher
cache and student states restored) through the public step API with the
per-step host-to-device copy of token ids from pinned memory and the
device-to-host read of every step's loss metrics inside the timed region; the
read of step s completes after step s + 1 is issued, and the last step's read
completes before the clock stops.

--impl reference runs the unmodified reference package (installed under
baseline/_ref) through its own API on the same synthetic data.
"""
import argparse
import copy
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
BASELINE_TOKENS_PER_S = None  # the reference project publishes no throughput figure for this config

MODEL_27B = dict(vocab_size=248077, hidden_size=5120, intermediate_size=17408, num_hidden_layers=64,
                 num_attention_heads=24, num_key_value_heads=4, head_dim=256, linear_num_key_heads=16,
                 linear_num_value_heads=48, linear_key_head_dim=128, linear_value_head_dim=128,
                 linear_conv_kernel_dim=4, rms_norm_eps=1e-6, rope_theta=10000000.0, partial_rotary_factor=0.25)
MODEL_SMALL = dict(vocab_size=4096, hidden_size=1024, intermediate_size=2048, num_hidden_layers=8,
                   num_attention_heads=8, num_key_value_heads=2, head_dim=128, linear_num_key_heads=4,
                   linear_num_value_heads=8, linear_key_head_dim=128, linear_value_head_dim=128,
                   linear_conv_kernel_dim=4, rms_norm_eps=1e-6, rope_theta=10000000.0, partial_rotary_factor=0.25)


def layer_types(n):
    return ["full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(n)]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--model", choices=("27b", "small"), default="27b")
    p.add_argument("--chunk", type=int, default=1024)
    p.add_argument("--context", type=int, default=4096)
    p.add_argument("--micro-batch", type=int, default=1)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--overlap-students", type=int, choices=(0, 1), default=1,
                   help="ours: run the students' micro-steps on their own stream beside the teacher forward")
    p.add_argument("--profile", action="store_true", help="print a per-kernel breakdown of one step and exit")
    return p.parse_args()


# ---------------------------------------------------------------------------- environment
def init_env(args):
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", str(max(1, args.gpus if "LOCAL_RANK" in os.environ else 1)))
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("LOCAL_WORLD_SIZE", os.environ["WORLD_SIZE"])
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
    os.environ.setdefault("TQDM_DISABLE", "1")


def write_dataset(root, vocab, tokens_needed, seed):
    """Synthetic manifest v1: documents with log-uniform lengths in [256, 16384]."""
    import numpy as np
    from rwkv_theseus_b200.data import sha256_of_file
    rng = np.random.default_rng(seed)
    lengths, total = [], 0
    while total < tokens_needed:
        n = int(np.exp(rng.uniform(np.log(256), np.log(16384))))
        lengths.append(n)
        total += n
    root.mkdir(parents=True, exist_ok=True)
    rng.integers(0, vocab, size=total, dtype=np.uint32).astype("<u4").tofile(root / "tokens.bin")
    np.save(root / "offsets.npy", np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64))
    manifest = {"format": 1, "vocab_size": vocab, "sources": [{
        "tokens": "tokens.bin", "offsets": "offsets.npy", "weight": 1.0,
        "tokens_sha256": sha256_of_file(root / "tokens.bin"), "offsets_sha256": sha256_of_file(root / "offsets.npy")}]}
    (root / "manifest.json").write_text(json.dumps(manifest))
    return root / "manifest.json"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of this rank's GPU during the timed region."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, uuid):
        self.proc = None
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", uuid, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, flag in zip(self.NAMES, parts[3:7]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- our implementation
def build_ours(args, topo, manifest, model_spec):
    import torch
    from rwkv_theseus_b200.config import make_config
    from rwkv_theseus_b200.data import reader_for
    from rwkv_theseus_b200.models.hf_io import random_model
    from rwkv_theseus_b200.models.qwen35 import HybridConfig
    from rwkv_theseus_b200.models.runner import Capture, Runner, migration_order
    from rwkv_theseus_b200.stage import Student
    from rwkv_theseus_b200.trainer import StepEngine
    mcfg = HybridConfig(**model_spec, layer_types=layer_types(model_spec["num_hidden_layers"]))
    model = random_model(mcfg, topo.device, seed=0)
    order = migration_order(model, len([t for t in mcfg.layer_types if t == "full_attention"]))
    cfg = make_config({"train_manifest": str(manifest), "validation_manifest": str(manifest),
                       "output": str(Path(tempfile.gettempdir()) / "bench_out"), "model": str(ROOT),
                       "chunk_tokens": args.chunk, "context_tokens": args.context,
                       "micro_batch_size": args.micro_batch, "training_mode": "epoch", "head_size": 64,
                       "backend": "cuda", "distributed_backend": "nccl",
                       "overlap_students": bool(args.overlap_students)})
    runner = Runner(model)
    students, captures = {}, {}
    for i, layer in enumerate(order):
        torch.manual_seed(cfg["seed"] + i)
        students[layer] = Student(mcfg, layer, cfg, topo, total_steps=10 ** 6)
        captures[layer] = Capture(model.model.layers[layer].self_attn)
    engine = StepEngine(cfg, topo, runner, order, students, captures)
    reader = reader_for(cfg, topo)

    pending = []

    def step(read):
        """One step; with `read` the step's metrics are started towards the host and the previous step's are
        read and validated (the host issues step s + 1 before it waits for step s's metrics)."""
        before = reader.consumed_tokens
        reports = engine.step(reader)
        if read:
            pending.append(engine.read_metrics_async(reports))
            if len(pending) > 1:
                pending.pop(0).result()
        return reader.consumed_tokens - before

    def finish():
        while pending:
            pending.pop(0).result()

    def phases():
        """Milliseconds per phase kind of one extra, untimed step: device time between CUDA events on the compute
        stream (updates: the enqueue on that stream of the previous step's updates, which run on a side stream
        under the teacher phase) and host time spent issuing the phase, plus the whole step's device time."""
        engine.profiler.on = True
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        try:  # a steady-state step: the previous step's updates are issued under its teacher forward
            start.record()
            reports = engine.step(reader)
            engine.join_students()  # stop after the step's last micro-steps (the step itself does not wait for them)
            stop.record()
            dev, host = engine.profiler.summary(), engine.profiler.host_summary()
            stop.synchronize()
            engine.read_metrics(reports)  # the phase step is validated like every other (faults, exchange status)
        finally:
            engine.profiler.on = False
        if topo.world > 1:  # every rank's split, for skew between ranks
            print(json.dumps({"rank": topo.rank, "phases_dev_ms": {k: round(v, 3) for k, v in dev.items()},
                              "phases_host_ms": {k: round(v, 3) for k, v in host.items()}}), file=sys.stderr,
                  flush=True)
        out = {"step_ms": start.elapsed_time(stop)}
        for key, prefix in (("teacher", "teacher"), ("students", "student_"), ("updates", "update_")):
            out[f"{key}_ms"] = sum(v for k, v in dev.items() if k.startswith(prefix))
            out[f"{key}_host_ms"] = sum(v for k, v in host.items() if k.startswith(prefix))
        return {k: round(v, 3) for k, v in out.items()}
    def snapshot():
        """Reader position, teacher cache and student states, so that the e2e pass replays the timed batches."""
        states = {layer: None if st.state is None else {k: v.clone() for k, v in st.state.items()}
                  for layer, st in students.items()}
        return copy.deepcopy(reader.state_dict()), runner.state_dict(), states

    def restore(snap):
        reader.load_state_dict(copy.deepcopy(snap[0]))
        runner.load_state_dict(snap[1])
        for layer, state in snap[2].items():
            students[layer].state = state
    def set_overlap(on):
        for student in students.values():
            student.overlap_update = on

    def profiled(on):
        engine.profiler.on = on
    step.finish = finish
    step.flush_updates = engine.join_updates  # issue the last step's updates; the current stream waits for them
    step.phases = phases
    step.snapshot, step.restore = snapshot, restore
    step.set_overlap, step.profiled = set_overlap, profiled
    return step


# ---------------------------------------------------------------------------- reference implementation
def reference_teacher(model_spec, device):
    """Random-init HF ``Qwen3_5ForCausalLM`` of the spec (bf16, frozen, sdpa attention): the teacher the unmodified
    reference package runs on (as its own tests construct it; the reference's ``load_model`` needs a checkpoint)."""
    import torch
    from transformers import Qwen3_5TextConfig, Qwen3_5ForCausalLM
    spec = dict(model_spec)
    theta, partial = spec.pop("rope_theta"), spec.pop("partial_rotary_factor")
    tcfg = Qwen3_5TextConfig(**spec, layer_types=layer_types(spec["num_hidden_layers"]),
                             rope_parameters={"rope_type": "default", "rope_theta": theta,
                                              "partial_rotary_factor": partial, "mrope_section": [11, 11, 10]})
    tcfg._attn_implementation = "sdpa"
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(device):
        model = Qwen3_5ForCausalLM(tcfg)
    torch.set_default_dtype(torch.float32)
    return model.requires_grad_(False).eval()


def build_reference(args, topo_unused, manifest, model_spec):
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    import torch
    from theseus.config import DEFAULTS
    from theseus.distributed import Topology
    from theseus.hf_model import Capture, Runner, migration_order
    from theseus.losses import statistics, metrics
    from theseus.stage import prepare_student
    from theseus.timemix import detach_state
    from theseus.validation import reader_for
    topo = Topology("nccl", 30)
    model = reference_teacher(model_spec, topo.device)
    tcfg = model.config
    order = migration_order(model, len([t for t in tcfg.layer_types if t == "full_attention"]))
    cfg = DEFAULTS | {"train_manifest": str(manifest), "validation_manifest": str(manifest), "head_size": 64,
                      "chunk_tokens": args.chunk, "context_tokens": args.context,
                      "micro_batch_size": args.micro_batch, "training_mode": "epoch", "backend": "cuda",
                      "distributed_backend": "nccl"}
    runner = Runner(model)
    reader = reader_for(cfg, topo)
    students, captures = {}, {}
    for index, layer in enumerate(order):
        torch.manual_seed(cfg["seed"] + index)
        students[layer] = prepare_student(model, layer, cfg, topo, None, total_steps=10 ** 6, detached=True)
        captures[layer] = Capture(model.model.layers[layer].self_attn)

    def step(read, mark=None):
        # The body of the reference train.py step loop (train.py:153-211) with grad_accum_steps = 1. `mark(kind)`
        # (phase split only) records a CUDA event at the start of each phase of that kind.
        mark = mark or (lambda kind: None)
        accum = {layer: torch.zeros(3, device=topo.device) for layer in order}
        for _, _, optimizer, _ in students.values():
            optimizer.zero_grad(set_to_none=True)
        batch = reader.next()
        if batch["reset"]:
            runner.reset()
            for adapter, *_ in students.values():
                adapter.state = None
        mark("teacher")
        runner.forward(batch["ids"].to(topo.device))
        for layer in order:
            mark("students")
            adapter, ddp, optimizer, scheduler = students[layer]
            capture = captures[layer]
            x, target = capture.x, capture.y
            with torch.autocast(topo.device.type, dtype=torch.bfloat16):
                prediction, state = ddp(x, adapter.state)
            adapter.state = detach_state(state)
            stats = statistics(prediction, target, cfg["loss_epsilon"])
            accum[layer] += stats.detach()
            stats[0].backward()
            del prediction, state, stats, x, target
            capture.x = capture.y = None
            mark("updates")
            topo.student_sum(accum[layer])
            count = accum[layer][2]
            if count.item() <= 0:
                raise RuntimeError("No training tokens in update")
            for p in adapter.core.parameters():
                if p.grad is not None:
                    p.grad.mul_(topo.world / count)
            norm = torch.nn.utils.clip_grad_norm_(adapter.core.parameters(), cfg["clip_norm"],
                                                  error_if_nonfinite=True)
            optimizer.step()
            scheduler.step()
            optimizer.zero_grad(set_to_none=True)
            if read:
                metrics(accum[layer]) | {"grad_norm": norm.item()}
        mark("end")
        return int(batch["ids"].numel())

    def phases():
        """Device ms per phase kind of one extra, untimed step, between CUDA events recorded on the reference's
        stream at each phase start: teacher forward, student forward + backward (with DDP's gradient all-reduce,
        which runs inside backward), and the update (metric sum, gradient scale, clip, AdamW, scheduler). The same
        keys as this package's split."""
        marks = []

        def mark(kind):
            event = torch.cuda.Event(enable_timing=True)
            event.record()
            marks.append((kind, event))
        step(False, mark)
        torch.cuda.synchronize(topo.device)
        out = {"step_ms": marks[0][1].elapsed_time(marks[-1][1])}
        for kind in ("teacher", "students", "updates"):
            out[f"{kind}_ms"] = sum(a.elapsed_time(b) for (k, a), (_, b) in zip(marks, marks[1:]) if k == kind)
        return {k: round(v, 3) for k, v in out.items()}
    step.phases = phases
    return step, topo


# ---------------------------------------------------------------------------- driver
# Name fragments of this package's kernels (csrc/); everything else in a trace is a library or ATen kernel.
OWN_KERNELS = ("wkv7_", "gemm_kernel", "rmsnorm_", "conv1d_silu", "gdn_", "mix_kernel", "mix_bwd", "pre_wkv",
               "post_wkv", "nmse_loss", "adamw_kernel", "scale_norm", "act_kernel", "act_bwd", "norm_rope",
               "copy_rows", "to_bf16", "report_kernel", "gated_rmsnorm", "flash_attn", "exchange_", "loss_rows",
               "norm2_kernel", "skinny_", "kl_", "zero_f32", "copy_bytes", "mix_vec", "embed_rows")


def count_launches(step_fn):
    """Kernels launched by one step, split into this package's kernels and others (profiled, untimed)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    mine = OWN_KERNELS
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn(False)
        torch.cuda.synchronize()
    ours = other = 0
    names = {}
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA:
            continue
        if any(key in evt.name for key in mine):
            ours += 1
        else:
            other += 1
            names[evt.name[:60]] = names.get(evt.name[:60], 0) + 1
    return ours, other, names


def kernel_group(name):
    """Kernel name without parameters and namespaces; GEMMs keep their tile width and epilogue code."""
    if name.startswith("Memcpy") or name.startswith("Memset"):
        return name.split(" ")[0]
    plain = name.replace("(anonymous namespace)::", "")
    head = (plain[5:] if plain.startswith("void ") else plain).split("(")[0]
    if "gemm_kernel<" in name:
        args = name.split("gemm_kernel<", 1)[1].split(">")[0].split(",")
        return f"gemm_kernel<BN {args[0].strip()}, EPI {args[-1].strip()}>"
    head = head.split("<")[0]
    return head.rsplit("::", 1)[-1] or name[:60]


def print_breakdown(step_fn, rank):
    """Per-kernel device time of one step, grouped by kernel name, then by step phase (profiled; not a benchmark
    number). Also the phase split of one step with the optimizer updates overlapped (the default) and serial."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    if hasattr(step_fn, "phases"):
        snap = step_fn.snapshot()  # both splits and the profiled step run the same batch
        overlapped = step_fn.phases()
        step_fn.restore(snap)
        snap = step_fn.snapshot()
        step_fn.set_overlap(False)
        serial = step_fn.phases()
        step_fn.set_overlap(True)
        step_fn.restore(snap)
        if rank == 0:
            print("phases, updates overlapped:", json.dumps(overlapped))
            print("phases, updates serial:    ", json.dumps(serial))
    if hasattr(step_fn, "profiled"):
        step_fn.profiled(True)
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        step_fn(False)  # steady state: the previous step's updates run under this step's teacher forward
        torch.cuda.synchronize()
    if hasattr(step_fn, "profiled"):
        step_fn.profiled(False)
    groups = {}
    total = 0.0
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA or evt.name.startswith("phase:"):
            continue
        name = kernel_group(evt.name)
        dur = evt.device_time_total if hasattr(evt, "device_time_total") else evt.cuda_time_total
        groups[name] = groups.get(name, [0.0, 0])
        groups[name][0] += dur
        groups[name][1] += 1
        total += dur
    if rank == 0:
        for name, (us, n) in sorted(groups.items(), key=lambda kv: -kv[1][0])[:30]:
            print(f"{us / 1000:9.3f} ms {100 * us / total:5.1f}% {n:6d}  {name[:90]}")
        print(f"{total / 1000:9.3f} ms total kernel time")
        print_timeline(prof)
        print_phase_kernels(prof)
        print_host_api(prof)


def print_host_api(prof):
    """Host time spent inside CUDA runtime/driver calls during the profiled step, by call name (how much of the
    host's issue time the API calls themselves take, against the Python and C++ code around them)."""
    import torch
    cpu = torch.autograd.DeviceType.CPU
    calls = {}
    for e in prof.profiler.kineto_results.events():
        name = e.name()
        if e.device_type() != cpu or not name.startswith("cu"):
            continue
        entry = calls.setdefault(name, [0, 0])
        entry[0] += e.duration_ns()
        entry[1] += 1
    total = sum(ns for ns, _ in calls.values())
    print(f"host API calls: {total / 1e6:.3f} ms in {sum(n for _, n in calls.values())} calls")
    for name, (ns, n) in sorted(calls.items(), key=lambda kv: -kv[1][0])[:12]:
        print(f"    {ns / 1e6:8.3f} ms {n:6d}  {name[:70]}")


def print_phase_kernels(prof):
    """Kernel time per step phase: each kernel is charged to the innermost ``phase:`` range that contains the host
    call that launched it (the launch's correlation id; a CUDA graph replay charges all its kernels)."""
    import torch
    cpu, cuda = torch.autograd.DeviceType.CPU, torch.autograd.DeviceType.CUDA
    events = prof.profiler.kineto_results.events()
    ranges = sorted((e.start_ns(), e.end_ns(), e.name()[6:]) for e in events
                    if e.device_type() == cpu and e.name().startswith("phase:"))
    launch_at = {e.correlation_id(): e.start_ns() for e in events
                 if e.device_type() == cpu and e.name().startswith("cuda")}
    per = {}
    for e in events:
        if e.device_type() != cuda or e.name().startswith("phase:") or e.duration_ns() <= 0:
            continue
        at = launch_at.get(e.correlation_id())
        phase = "other"
        if at is not None:
            inside = [r for r in ranges if r[0] <= at <= r[1]]
            if inside:
                name = min(inside, key=lambda r: r[1] - r[0])[2]
                phase = name.split("_")[0]
        kinds = per.setdefault(phase, {})
        group = kernel_group(e.name())
        kinds[group] = kinds.get(group, 0) + e.duration_ns()
    for phase, kinds in sorted(per.items(), key=lambda kv: -sum(kv[1].values())):
        print(f"phase {phase}: {sum(kinds.values()) / 1e6:.3f} ms of kernels")
        for group, ns in sorted(kinds.items(), key=lambda kv: -kv[1])[:12]:
            print(f"    {ns / 1e6:8.3f} ms  {group[:80]}")
        foreign = {}
        for e in events:
            if e.device_type() != cuda or e.duration_ns() <= 0 or any(k in e.name() for k in OWN_KERNELS):
                continue
            at = launch_at.get(e.correlation_id())
            inside = [r for r in ranges if at is not None and r[0] <= at <= r[1]]
            name = min(inside, key=lambda r: r[1] - r[0])[2].split("_")[0] if inside else "other"
            if name == phase and not e.name().startswith("phase:"):
                foreign[e.name()[:90]] = foreign.get(e.name()[:90], 0) + 1
        for name, n in sorted(foreign.items(), key=lambda kv: -kv[1])[:8]:
            print(f"    library/ATen x{n}: {name}")


def print_timeline(prof):
    """Busy time per stream, the step's span and the largest idle gaps of the device (all streams together)."""
    import torch
    spans = []
    for e in prof.profiler.kineto_results.events():
        if e.device_type() != torch.autograd.DeviceType.CUDA or e.duration_ns() <= 0 or e.name().startswith("phase:"):
            continue
        spans.append((e.start_ns(), e.end_ns(), e.device_resource_id(), kernel_group(e.name())))
    if not spans:
        return
    spans.sort()
    t0, t1 = spans[0][0], max(s[1] for s in spans)
    busy = {}
    for stream in {s[2] for s in spans}:
        end, total = 0, 0
        for a, b, st, _ in spans:
            if st != stream:
                continue
            a = max(a, end)
            if b > a:
                total += b - a
                end = b
        busy[stream] = total
    gaps, end, before = [], spans[0][1], spans[0][3]
    for a, b, _, name in spans[1:]:
        if a > end:
            gaps.append((a - end, before, name))
        if b > end:
            end, before = b, name
    print(f"step span {(t1 - t0) / 1e6:.3f} ms; busy per stream (ms): "
          + ", ".join(f"{st}: {ns / 1e6:.3f}" for st, ns in sorted(busy.items(), key=lambda kv: -kv[1])))
    print(f"device idle {sum(g[0] for g in gaps) / 1e6:.3f} ms in {len(gaps)} gaps; largest:")
    for ns, a, b in sorted(gaps, reverse=True)[:12]:
        print(f"  {ns / 1e3:9.1f} us  after {a[:40]}  before {b[:40]}")


def main():
    args = parse()
    init_env(args)
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if args.impl == "reference" and not (ROOT / "baseline" / "_ref" / "theseus").exists():
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    model_spec = MODEL_27B if args.model == "27b" else MODEL_SMALL
    needed = (args.warmup + 2 * args.steps + 16) * args.chunk * args.micro_batch * 2
    data_root = Path(tempfile.gettempdir()) / f"theseus_bench_{os.environ.get('MASTER_PORT')}_{rank}"
    topo = None
    if args.impl == "ours":
        from rwkv_theseus_b200.parallel.topology import Topology
        topo = Topology("nccl", 30)
        manifest = write_dataset(data_root, model_spec["vocab_size"], needed * world, seed=1234)
        step = build_ours(args, topo, manifest, model_spec)
        device = topo.device
    else:
        manifest = write_dataset(data_root, model_spec["vocab_size"], needed * world, seed=1234)
        step, topo = build_reference(args, None, manifest, model_spec)
        device = topo.device

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    if args.profile:
        for _ in range(args.warmup):
            step(False)
        barrier()
        print_breakdown(step, rank)
        return
    # Start the clock sampler before warm-up: nvidia-smi's start-up briefly stalls CUDA calls.
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    sampler = ClockSampler(uuid)
    time.sleep(2.0)
    for _ in range(args.warmup):
        step(False)
    if hasattr(step, "flush_updates"):
        step.flush_updates()  # the last warm-up step's updates finish before the timed region
    snap = step.snapshot() if hasattr(step, "snapshot") else None
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record()
    tokens = 0
    for _ in range(args.steps):
        tokens += step(False)
    if hasattr(step, "flush_updates"):
        step.flush_updates()  # the K-th step's updates are inside the timed region (stop waits for them)
    stop.record()
    barrier()
    clocks = sampler.stop()
    ms = start.elapsed_time(stop)
    e2e_ms = None
    e2e_tokens = 0
    if not args.no_e2e:
        if snap is not None:
            step.restore(snap)  # the e2e pass runs the same K batches as the device-timed pass
            del snap
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_tokens += step(True)
        if hasattr(step, "finish"):
            step.finish()  # the last step's metrics, inside the timed region
        barrier()
        e2e_ms = (time.perf_counter() - t0) * 1000
    stats = torch.tensor([ms, float(tokens), e2e_ms or 0.0, float(e2e_tokens)], device=device, dtype=torch.float64)
    if world > 1:
        gathered = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(gathered, stats)
    else:
        gathered = [stats]
    ms_max = max(g[0].item() for g in gathered)
    total_tokens = sum(g[1].item() for g in gathered)
    e2e_max = max(g[2].item() for g in gathered)
    e2e_total = sum(g[3].item() for g in gathered)
    phases = step.phases() if hasattr(step, "phases") else None
    ours_launches, other_launches, other_names = count_launches(step) if args.impl == "ours" else (0, 0, {})
    value = total_tokens / (ms_max / 1000)
    if rank == 0:
        line = {
            "metric": "train tokens/s (27B hybrid parallel layer migration, 16 TimeMix students)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / BASELINE_TOKENS_PER_S) if BASELINE_TOKENS_PER_S else None,
            "dtype": "bf16", "data": "synthetic (log-uniform docs 256..16384, uniform ids; random-init weights)",
            "config": {"model": f"qwen3.5-hybrid-{args.model} + 16 RWKV7 TimeMix students", "global_batch":
                       args.micro_batch * world, "seq_len": args.chunk, "context": args.context,
                       "parallelism": f"dp{world}", "tokens_timed": total_tokens,
                       "l2": "no flush: 54 GB of teacher weights streamed per step (> L2)"},
            "clocks": clocks,
            "e2e": None if args.no_e2e else {
                "value": e2e_total / (e2e_max / 1000), "unit": "tokens/s",
                "ms_per_step": e2e_max / args.steps, "tokens_timed": e2e_total,
                "batches": "the device-timed K batches again" if args.impl == "ours" else "the next K batches",
                "h2d_bytes_per_step": 8 * args.chunk * args.micro_batch,
                # ours: 16 reports of 5 fp32, 3 fault words, 4 exchange status words (world > 1)
                "d2h_bytes_per_step": (4 * 5 * 16 + 4 * 3 + (16 if world > 1 else 0)) if args.impl == "ours"
                else 4 * 3 * 16},
            "phases_ms": phases,  # one extra untimed step (rank 0): device and host ms per phase kind
            "gpu_launches": ours_launches * args.steps,
            "other_launches_per_step": other_launches,
        }
        if args.impl == "reference":
            line["impl"] = "reference"
        else:
            line["other_kernels"] = dict(sorted(other_names.items(), key=lambda kv: -kv[1])[:8])
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
    if topo is not None and hasattr(topo, "close"):
        try:
            topo.close()
        except Exception:
            pass


if __name__ == "__main__":
    main()
