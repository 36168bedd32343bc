import torch

from rwkv_theseus_b200.models.timemix import TimeMix, detach_state, PARAM_ORDER, lora_ranks
from rwkv_theseus_b200.ops.wkv7 import reference


def test_schema_matches_reference_order_and_shapes():
    model = TimeMix(64, 3, 8, head_size=16, backend="reference")
    names = list(model.state_dict())
    assert tuple(names) == PARAM_ORDER and len(names) == 23
    assert model.w1.shape == (64, 32) and model.g2.shape == (32, 64) and model.r_k.shape == (4, 16)
    assert lora_ranks(5120) == (192, 352)
    assert lora_ranks(64, 8, 8) == (8, 8)


def test_streaming_output_and_state():
    model = TimeMix(32, 3, 8, head_size=8, backend="reference")
    torch.nn.init.normal_(model.output.weight, std=.03)
    x = torch.randn(2, 9, 32)
    full, end = model(x)
    a, state = model(x[:, :4])
    b, state = model(x[:, 4:], state)
    torch.testing.assert_close(torch.cat([a, b], 1), full)
    for key in state:
        torch.testing.assert_close(state[key], end[key])


def test_initialization_can_learn():
    model = TimeMix(32, 3, 8, head_size=8, backend="reference")
    opt = torch.optim.AdamW(model.parameters(), lr=.01)
    x, target = torch.randn(1, 5, 32), torch.randn(1, 5, 32)
    for step in range(3):
        opt.zero_grad()
        y, _ = model(x)
        (y - target).square().mean().backward()
        assert model.output.weight.grad.abs().sum() > 0
        if step:
            assert model.receptance.weight.grad.abs().sum() > 0
            assert model.g1.grad.abs().sum() > 0
        opt.step()


def test_tbptt_detaches_only_at_chunk_boundary():
    model = TimeMix(16, 1, 4, head_size=4, backend="reference")
    torch.nn.init.normal_(model.output.weight, std=.05)
    x1 = torch.randn(1, 3, 16, requires_grad=True)
    x2 = torch.randn(1, 4, 16, requires_grad=True)
    _, state = model(x1)
    y, _ = model(x2, detach_state(state))
    y.sum().backward()
    assert x1.grad is None
    assert x2.grad is not None and x2.grad.abs().sum() > 0


def test_reference_recurrence_matches_explicit_loop():
    torch.manual_seed(0)
    B, T, H, N = 2, 5, 2, 4
    r, w, k, v, a, b = [torch.randn(B, T, H, N) for _ in range(6)]
    s0 = torch.randn(B, H, N, N)
    y, end = reference(r, w, k, v, a, b, s0)
    s = s0.clone()
    for t in range(T):
        for bb in range(B):
            for h in range(H):
                d = torch.exp(-0.6065306597126334 * torch.sigmoid(w[bb, t, h]))
                S = s[bb, h]
                S = S * d[None] + (S @ a[bb, t, h])[:, None] * b[bb, t, h][None] + v[bb, t, h][:, None] * k[bb, t, h][None]
                s[bb, h] = S
                torch.testing.assert_close(y[bb, t, h], S @ r[bb, t, h], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(end, s, atol=1e-5, rtol=1e-5)
