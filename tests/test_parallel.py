"""The real training loop with an in-process stand-in topology (reference ``tests/test_parallel.py``):
one teacher forward per step, then each layer's forward/backward, reduction and update in migration
order before the next layer starts; the frozen teacher is untouched and gets no gradients."""
import json
from types import SimpleNamespace

import torch

from fixtures import make_config
from rwkv_theseus_b200 import trainer
from rwkv_theseus_b200.config import make_config as validated
from rwkv_theseus_b200.models.runner import AttentionAdapter, Runner
from rwkv_theseus_b200.stage import Student


def fake_topology():
    noop = lambda *args, **kwargs: None  # noqa: E731
    return SimpleNamespace(rank=0, leader=0, world=1, device=torch.device("cpu"), tracker=None,
                           student_group=None, assert_same=noop, barrier=noop, close=noop, synchronize=noop,
                           broadcast_object=lambda value, source=None: value, student_sum=lambda value: value,
                           grad_sync=lambda: None, join_grad_sync=noop, check_grad_sync=noop)


def test_one_teacher_forward_then_immediate_layer_updates(tmp_path, monkeypatch):
    raw, _ = make_config(tmp_path, 2)
    cfg = validated(raw | {"grad_accum_steps": 1, "original_teacher_kl": False})
    monkeypatch.setattr(trainer, "Topology", lambda *args: fake_topology())
    events, teachers = [], []
    load = trainer.load_model

    def load_model(*args, **kwargs):
        model = load(*args, **kwargs)
        teachers.append((model, {k: v.clone() for k, v in model.state_dict().items()}))
        return model
    monkeypatch.setattr(trainer, "load_model", load_model)
    forward = Runner.forward

    def teacher_forward(runner, ids, *args, **kwargs):
        assert not any(isinstance(m, AttentionAdapter) for m in runner.model.modules())
        assert not any(p.requires_grad for p in runner.model.parameters())
        events.append("teacher")
        return forward(runner, ids, *args, **kwargs)
    monkeypatch.setattr(Runner, "forward", teacher_forward)
    for method in ("micro_step", "reduce", "update"):
        original = getattr(Student, method)

        def wrapped(self, *args, _original=original, _name=method, **kwargs):
            if _name == "micro_step":
                x = args[0]
                assert not x.requires_grad and x.grad_fn is None  # detached teacher activations
            events.append((_name, self.layer))
            return _original(self, *args, **kwargs)
        monkeypatch.setattr(Student, method, wrapped)
    trainer.run(cfg, stop_after=1)
    assert events == ["teacher", ("micro_step", 1), ("reduce", 1), ("update", 1),
                      ("micro_step", 3), ("reduce", 3), ("update", 3)]
    model, before = teachers[0]
    for name, value in model.state_dict().items():
        torch.testing.assert_close(value, before[name], atol=0, rtol=0)
    assert all(p.grad is None for p in model.parameters())
    logs = [json.loads(line) for line in (tmp_path / "full" / "metrics.jsonl").read_text().splitlines()]
    train = next(item for item in logs if item["event"] == "train")
    assert train["sum_loss"] == sum(v["nmse"] for v in train["layers"].values())
    assert abs(train["mean_cos"] - sum(v["cosine"] for v in train["layers"].values()) / 2) < 1e-12
    assert not (tmp_path / "full" / "converted").exists()
