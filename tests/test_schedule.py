"""Learning-rate schedule: warmup, plateau and cosine phases, driven through torch's LambdaLR the way the
optimizer state dicts see it."""
import math

import pytest
import torch

from rwkv_theseus_b200.schedule import lr_at, lr_factor

CFG = dict(lr=2e-4, min_lr=1e-5, warmup_steps=40, constant_steps=60)


def closed_form(update, cfg, total):
    """The intended rate of optimizer update number `update` (1-based), written independently of lr_factor."""
    if update <= cfg["warmup_steps"]:
        return cfg["lr"] * update / cfg["warmup_steps"]
    knee = cfg["warmup_steps"] + cfg["constant_steps"]
    if update <= knee:
        return cfg["lr"]
    frac = min(1.0, (update - knee) / max(1, total - knee))
    return cfg["min_lr"] + (cfg["lr"] - cfg["min_lr"]) * (1 + math.cos(math.pi * frac)) / 2


@pytest.mark.parametrize("total", [7, 100, 101, 250])
def test_lambda_lr_follows_the_closed_form(total):
    param = torch.nn.Parameter(torch.zeros(()))
    opt = torch.optim.AdamW([param], lr=CFG["lr"])
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda n: lr_factor(n, CFG, total))
    for update in range(1, total + 1):
        assert opt.param_groups[0]["lr"] == pytest.approx(closed_form(update, CFG, total), rel=1e-9)
        assert lr_at(update - 1, CFG, total) == pytest.approx(opt.param_groups[0]["lr"], rel=1e-12)
        opt.step()
        sched.step()


def test_phase_shapes():
    total = 250
    rates = [lr_at(n, CFG, total) for n in range(total)]
    warm, flat, tail = rates[:40], rates[40:100], rates[100:]
    assert all(b > a for a, b in zip(warm, warm[1:])) and warm[-1] == pytest.approx(CFG["lr"])
    assert flat == [CFG["lr"]] * 60
    assert all(b <= a for a, b in zip(tail, tail[1:])) and tail[0] < CFG["lr"]
    assert tail[-1] == pytest.approx(CFG["min_lr"])
    mid = 100 + (total - 100) // 2 - 1   # the update halfway down the cosine
    assert rates[mid] == pytest.approx((CFG["lr"] + CFG["min_lr"]) / 2, rel=1e-2)


def test_runs_shorter_than_warmup_or_without_warmup_and_plateau():
    assert lr_factor(3, CFG, 5) == pytest.approx(4 / 40)          # still warming up at the last update
    assert lr_factor(69, CFG, 70) == 1.0                           # ends on the plateau
    bare = CFG | dict(warmup_steps=0, constant_steps=0)
    floor = CFG["min_lr"] / CFG["lr"]
    assert lr_factor(0, bare, 10) == pytest.approx(floor + (1 - floor) * (1 + math.cos(math.pi / 10)) / 2)
    assert lr_factor(9, bare, 10) == pytest.approx(floor)
