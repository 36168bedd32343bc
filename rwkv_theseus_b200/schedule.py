"""Learning-rate schedule (reference ``theseus/stage.py:8-20``).

Linear warmup to ``lr``, a constant plateau, then a cosine down to ``min_lr``.
``step_index`` is zero-based like ``LambdaLR``; the factor applies to the
*next* optimizer update.
"""
import math


def lr_factor(step_index, cfg, total_steps):
    update = step_index + 1
    warmup = cfg["warmup_steps"]
    plateau_end = warmup + cfg["constant_steps"]
    if update <= warmup:
        return update / warmup
    if update <= plateau_end:
        return 1.0
    # Stages shorter than warmup + plateau never reach the cosine phase.
    progress = min(1.0, (update - plateau_end) / max(1, total_steps - plateau_end))
    floor = cfg["min_lr"] / cfg["lr"]
    return floor + (1.0 - floor) * 0.5 * (1.0 + math.cos(math.pi * progress))


def lr_at(step_index, cfg, total_steps):
    return cfg["lr"] * lr_factor(step_index, cfg, total_steps)
