"""StepEngine on CUDA: per-layer updates deferred to the next step's start (the default) give the same training
trajectory as updates issued right after each layer's micro-step, and the asynchronous metric read returns the
same values as a synchronous one."""
import pytest
import torch

from rwkv_theseus_b200.config import DEFAULTS
from rwkv_theseus_b200.models.hf_io import random_model
from rwkv_theseus_b200.models.runner import Capture, Runner, migration_order
from rwkv_theseus_b200.smoke import smoke_config
from rwkv_theseus_b200.stage import Student
from rwkv_theseus_b200.trainer import StepEngine

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


class Topo:
    rank, world, leader = 0, 1, 0
    device = torch.device("cuda", 0)

    def grad_sync(self):
        return None


class Reader:
    """Fixed batches: a two-chunk document, then a new window."""

    def __init__(self, chunk, vocab, steps):
        g = torch.Generator().manual_seed(11)
        self.batches = []
        position = 0
        for step in range(steps):
            reset = step % 2 == 0
            position = 0 if reset else position + chunk
            self.batches.append({"ids": torch.randint(0, vocab, (1, chunk), generator=g), "reset": reset,
                                 "position": position})
        self.i = 0
        self.consumed_tokens = 0

    def next(self):
        batch = self.batches[self.i]
        self.i += 1
        self.consumed_tokens += batch["ids"].numel()
        return batch


def engine(defer, chunk, steps, overlap=True):
    cfg_model = smoke_config()
    model = random_model(cfg_model, torch.device("cuda"), seed=3)
    order = migration_order(model, 2)
    cfg = DEFAULTS | {"head_size": 64, "backend": "cuda", "lr": 1e-3, "warmup_steps": 0, "chunk_tokens": chunk,
                      "overlap_students": overlap}
    students, captures = {}, {}
    for i, layer in enumerate(order):
        torch.manual_seed(cfg["seed"] + i)
        students[layer] = Student(cfg_model, layer, cfg, Topo(), total_steps=10)
        captures[layer] = Capture(model.model.layers[layer].self_attn)
    eng = StepEngine(cfg, Topo(), Runner(model), order, students, captures)
    eng.defer_updates = defer
    return eng, Reader(chunk, cfg_model.vocab_size, steps)


@cuda
@pytest.mark.parametrize("chunk", [128, 96])  # 128: tcgen05 WKV7 path; 96: chunk-16 path (under 128 steps)
def test_deferred_updates_match_immediate(chunk):
    steps = 4
    runs = {}
    for defer in (True, False):
        eng, reader = engine(defer, chunk, steps)
        pending, logged = None, []
        for _ in range(steps):
            reports = eng.step(reader)
            if pending is not None:
                logged.append(pending.result())
            pending = eng.read_metrics_async(reports)
        logged.append(pending.result())
        eng.join_updates()
        torch.cuda.synchronize()
        runs[defer] = (eng, logged)
    (deferred, log_d), (immediate, log_i) = runs[True], runs[False]
    for layer in deferred.order:
        a, b = deferred.students[layer], immediate.students[layer]
        assert a.steps_done == b.steps_done == steps
        torch.testing.assert_close(a.flat.param, b.flat.param, rtol=1e-5, atol=1e-7)
        torch.testing.assert_close(a.flat.exp_avg_sq, b.flat.exp_avg_sq, rtol=1e-4, atol=1e-12)
    assert len(log_d) == len(log_i) == steps
    for md, mi in zip(log_d, log_i):
        assert md.keys() == mi.keys()
        for key in md:
            assert md[key]["tokens"] == mi[key]["tokens"]
            assert abs(md[key]["nmse"] - mi[key]["nmse"]) <= 1e-4 * abs(mi[key]["nmse"]) + 1e-7
            assert abs(md[key]["lr"] - mi[key]["lr"]) < 1e-12
    for eng in (deferred, immediate):
        for capture in eng.captures.values():
            capture.close()
    from rwkv_theseus_b200.ops import native
    native().gemm_set_concurrent(False)  # process-wide switch the overlapping engine turned on


def _train(eng, reader, steps):
    pending, logged = None, []
    for _ in range(steps):
        reports = eng.step(reader)
        if pending is not None:
            logged.append(pending.result())
        pending = eng.read_metrics_async(reports)
    logged.append(pending.result())
    eng.join_updates()
    torch.cuda.synchronize()
    return logged


@cuda
@pytest.mark.parametrize("chunk", [128, 96])
def test_students_beside_teacher_match_serial_schedule(chunk):
    """Students on their own stream (each waiting only for its layer's capture event) train exactly like students
    issued after the whole teacher forward on the compute stream."""
    from rwkv_theseus_b200.ops import native
    steps = 4
    try:
        runs = {}
        for overlap in (True, False):
            eng, reader = engine(True, chunk, steps, overlap=overlap)
            assert (eng.student_stream is not None) == overlap
            runs[overlap] = (eng, _train(eng, reader, steps))
        (side, log_s), (serial, log_c) = runs[True], runs[False]
        for layer in side.order:
            a, b = side.students[layer], serial.students[layer]
            torch.testing.assert_close(a.flat.param, b.flat.param, rtol=1e-5, atol=1e-6)
        for ms, mc in zip(log_s, log_c):
            for key in ms:
                assert ms[key]["tokens"] == mc[key]["tokens"]
                assert abs(ms[key]["nmse"] - mc[key]["nmse"]) <= 1e-3 * abs(mc[key]["nmse"]) + 1e-6
        for eng, _ in runs.values():
            for capture in eng.captures.values():
                capture.close()
    finally:
        native().gemm_set_concurrent(False)  # process-wide switch the overlapping engine turned on
