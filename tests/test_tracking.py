"""W&B tracker against a fake SDK module: leader-only start, resume identity, metric keys and steps
(the reference's ``tests/test_tracking.py`` contract)."""
import sys
from types import SimpleNamespace

import pytest

from rwkv_theseus_b200.config import DEFAULTS
from rwkv_theseus_b200.tracking import Tracker


class FakeWandb:
    def __init__(self, ids):
        self.inits, self.logged, self.finished, self.metrics = [], [], [], []
        self.util = SimpleNamespace(generate_id=lambda: next(ids))

    @staticmethod
    def Settings(**kwargs):  # noqa: N802 - mirrors the SDK's name
        return kwargs

    def init(self, **kwargs):
        self.inits.append(kwargs)
        fake = self

        class Run:
            def define_metric(self, name, **kw):
                assert "*" not in name[:-1], "only suffix globs are supported by W&B"
                fake.metrics.append((name, kw.get("step_metric")))

            def log(self, values):
                fake.logged.append(values)

            def finish(self, **kw):
                fake.finished.append(kw)
        return Run()


@pytest.mark.parametrize("mode", ["online", "offline"])
def test_leader_only_resume_and_metric_keys(tmp_path, monkeypatch, mode):
    ids = iter(["run1", "run2", "run3"])
    sdk = FakeWandb(ids)
    monkeypatch.setattr("rwkv_theseus_b200.tracking.uuid4", lambda: SimpleNamespace(hex=next(ids)))
    monkeypatch.setitem(sys.modules, "wandb", sdk)
    cfg = DEFAULTS | {"output": str(tmp_path), "wandb_mode": mode}
    tracker = Tracker()
    tracker.start(cfg, SimpleNamespace(rank=1, leader=0))
    assert not sdk.inits  # non-leaders never start a run
    tracker.start(cfg, SimpleNamespace(rank=0, leader=0))
    assert sdk.inits[0]["mode"] == mode and sdk.inits[0]["resume"] is None
    assert ("sum_loss", "progress/global_step") in sdk.metrics
    layers = {"layer_03": {"nmse": 0.4, "cosine": 0.8, "rrms": 0.4 ** 0.5, "lr": 1e-3, "grad_norm": 2.0}}
    tracker.log("train", {"step": 5, "sum_loss": 0.4, "mean_cos": 0.8, "layers": layers})
    tracker.log("validation", {"step": 5, "sum_loss": 0.3, "mean_cos": 0.9,
                               "layers": {"layer_03": {"nmse": 0.3, "rrms": 0.3 ** 0.5, "cosine": 0.9}}})
    tracker.log("checkpoint", {"path": "x"})  # not a tracked event
    train, val = sdk.logged
    assert train["progress/global_step"] == val["progress/global_step"] == 5
    assert (train["sum_loss"], train["mean_cos"], train["layer_03/grad_norm"]) == (0.4, 0.8, 2.0)
    assert val["val/layer_03/cosine"] == 0.9 and val["val/sum_loss"] == 0.3
    assert {k for k in train if "/" not in k} == {"sum_loss", "mean_cos"}
    tracker.finish()
    tracker.start(cfg, SimpleNamespace(rank=0, leader=0), resume=True)
    first_id = sdk.inits[0]["id"]
    if mode == "online":  # an online run resumes under its recorded id
        assert sdk.inits[1]["id"] == first_id and sdk.inits[1]["resume"] == "allow"
    else:
        assert sdk.inits[1]["id"] != first_id and sdk.inits[1]["resume"] is None
    tracker.finish(exit_code=1)
    assert sdk.finished == [{"exit_code": 0}, {"exit_code": 1}]


def test_disabled_mode_never_imports_the_sdk(monkeypatch):
    monkeypatch.setitem(sys.modules, "wandb", None)  # importing it would raise
    tracker = Tracker()
    tracker.start(DEFAULTS, SimpleNamespace(rank=0, leader=0))
    tracker.log("train", {})
    tracker.finish()
