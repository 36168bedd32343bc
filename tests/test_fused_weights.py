"""Fused teacher projection weights (ops.gdn.fused_weight): one buffer, parameters re-pointed to views."""
import torch
from torch import nn

from rwkv_theseus_b200.ops.gdn import fused_weight


def _module(dtype):
    torch.manual_seed(0)
    m = nn.Module()
    m.a = nn.Linear(16, 8, bias=False)
    m.b = nn.Linear(16, 4, bias=False)
    m.c = nn.Linear(16, 2, bias=False)
    m.to(dtype).requires_grad_(False)
    return m


def test_frozen_bf16_parameters_become_views_of_the_fused_weight():
    m = _module(torch.bfloat16)
    before = {k: v.clone() for k, v in m.state_dict().items()}
    w = fused_weight(m, ("a", "b", "c"), "_w")
    assert w.shape == (14, 16) and w.is_contiguous()
    assert torch.equal(w, torch.cat([before["a.weight"], before["b.weight"], before["c.weight"]]))
    for name in ("a", "b", "c"):
        p = getattr(m, name).weight
        assert p.untyped_storage().data_ptr() == w.untyped_storage().data_ptr()  # no second copy
        assert torch.equal(p, before[f"{name}.weight"])
    assert fused_weight(m, ("a", "b", "c"), "_w") is w  # built once
    x = torch.randn(3, 16).to(torch.bfloat16)
    y = x.float() @ w.float().t()
    torch.testing.assert_close(y[:, 8:12], x.float() @ m.b.weight.float().t())


def test_trainable_or_fp32_parameters_keep_their_own_storage():
    m = _module(torch.float32)
    w = fused_weight(m, ("a", "b"), "_w")
    assert w.dtype == torch.bfloat16
    assert m.a.weight.dtype == torch.float32
    assert m.a.weight.untyped_storage().data_ptr() != w.untyped_storage().data_ptr()
