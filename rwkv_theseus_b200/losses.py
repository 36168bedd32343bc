"""Distillation statistics (reference ``theseus/losses.py:5-30``).

``statistics`` returns the differentiable sums ``[sum NMSE, sum cosine, count]``
over tokens, with per-token NMSE = mean((x-y)^2) / max(mean(y^2), eps). On CUDA
the fused loss kernel computes the same three sums in one pass (and the NMSE
gradient in the same kernel, see ``ops.loss``); this module is the
device-agnostic definition used on CPU and as the test oracle.
"""
import math

import torch
from torch.nn import functional as F


def statistics(prediction, target, epsilon=1e-6, mask=None):
    x, y = prediction.float(), target.float()
    nmse = (x - y).square().mean(-1) / y.square().mean(-1).clamp_min(epsilon)
    cosine = F.cosine_similarity(x, y, dim=-1, eps=epsilon)
    weight = torch.ones_like(nmse) if mask is None else mask.float()
    return torch.stack([(nmse * weight).sum(), (cosine * weight).sum(), weight.sum()])


def loss_sum(stats, cosine_weight):
    """Training objective of summed statistics: sum NMSE + w * (token count - sum cosine)."""
    nmse_total, cos_total, count = stats[0], stats[1], stats[2]
    return nmse_total + cosine_weight * (count - cos_total)


def metrics(stats):
    """Per-token means of summed statistics: NMSE, its root (RRMS), cosine, and the token count."""
    totals = [float(v) for v in stats.detach().double().cpu()]
    tokens = totals[2]
    if not tokens > 0:
        raise ValueError("No valid validation tokens")
    per_token = totals[0] / tokens
    return {"nmse": per_token, "rrms": math.sqrt(per_token), "cosine": totals[1] / tokens, "tokens": int(tokens)}


def kl_sum(student_logits, teacher_logits):
    """Sum over tokens of KL(teacher || student) on the full vocabulary.

    CUDA tensors take the one-pass kernel (``csrc/fused/kl.cu``: online max / sums per row, per-row results
    summed here in a fixed order); otherwise two log_softmax passes (reference ``theseus/losses.py:27-30``)."""
    if student_logits.is_cuda:
        from .ops import native
        V = student_logits.shape[-1]
        s = student_logits.reshape(-1, V)
        t = teacher_logits.reshape(-1, V)
        if s.dtype not in (torch.bfloat16, torch.float32) or s.dtype != t.dtype:
            s, t = s.float(), t.float()
        return native().kl_rows(s.contiguous(), t.contiguous()).sum()
    teacher = F.log_softmax(teacher_logits.float(), dim=-1)
    student = F.log_softmax(student_logits.float(), dim=-1)
    return (teacher.exp() * (teacher - student)).sum()
