import pytest
import torch

from rwkv_theseus_b200.models.timemix import PARAM_ORDER, TimeMix, detach_state, lora_ranks
from rwkv_theseus_b200.ops.wkv7 import reference


def _mixer(width=32, layer=3, layers=8, head=8, seed=0, out_std=0.03):
    torch.manual_seed(seed)
    model = TimeMix(width, layer, layers, head_size=head, backend="reference")
    torch.nn.init.normal_(model.output.weight, std=out_std)  # the RWKV7 init zeroes it: every output would be 0
    return model


def test_schema_matches_reference_order_and_shapes():
    model = TimeMix(64, 3, 8, head_size=16, backend="reference")
    names = list(model.state_dict())
    assert tuple(names) == PARAM_ORDER and len(names) == 23
    assert model.w1.shape == (64, 32) and model.g2.shape == (32, 64) and model.r_k.shape == (4, 16)
    assert lora_ranks(5120) == (192, 352)
    assert lora_ranks(64, 8, 8) == (8, 8)


@pytest.mark.parametrize("cuts", [(1,), (5, 6), (2, 7, 10)])
def test_chunked_calls_equal_one_call(cuts):
    """Carrying (shift, wkv) across any split of a sequence reproduces the one-call output and end state."""
    model = _mixer(seed=len(cuts))
    x = torch.randn(3, 11, 32)
    whole, whole_end = model(x)
    pieces, state, start = [], None, 0
    for stop in (*cuts, x.shape[1]):
        y, state = model(x[:, start:stop], state)
        pieces.append(y)
        start = stop
    torch.testing.assert_close(torch.cat(pieces, 1), whole, rtol=1e-5, atol=1e-6)
    assert set(state) == set(whole_end) == {"shift", "wkv"}
    for key in state:
        torch.testing.assert_close(state[key], whole_end[key], rtol=1e-5, atol=1e-6)


def test_regression_loss_falls_and_reaches_the_projections():
    """A few AdamW steps on a fixed target lower the loss, and after the first step the gradient reaches the
    r/k/v projections and every LoRA branch (the zero-initialised output projection gates them at step 0)."""
    torch.manual_seed(1)
    model = TimeMix(32, 2, 6, head_size=8, backend="reference")
    opt = torch.optim.AdamW(model.parameters(), lr=0.02)
    x, target = torch.randn(2, 6, 32), torch.randn(2, 6, 32)
    losses = []
    for _ in range(6):
        opt.zero_grad()
        y, _ = model(x)
        loss = (y - target).square().mean()
        loss.backward()
        losses.append(loss.item())
        opt.step()
    assert losses[-1] < losses[0]
    for name in ("receptance.weight", "key.weight", "value.weight", "w1", "w2", "a1", "a2", "g1", "g2"):
        assert dict(model.named_parameters())[name].grad.abs().sum() > 0, name


def test_detached_state_cuts_the_graph_between_chunks():
    model = _mixer(width=16, layer=1, layers=4, head=4, out_std=0.05)
    first = torch.randn(1, 3, 16, requires_grad=True)
    second = torch.randn(1, 4, 16, requires_grad=True)
    _, state = model(first)
    carried, _ = model(second, state)             # state kept in the graph: the gradient reaches `first`
    (grad_first,) = torch.autograd.grad(carried.sum(), first, retain_graph=True)
    assert grad_first.abs().sum() > 0
    cut, _ = model(second, detach_state(state))   # detached: only the current chunk's input gets a gradient
    cut.sum().backward()
    assert first.grad is None
    assert second.grad is not None and second.grad.abs().sum() > 0


def test_reference_recurrence_matches_batched_token_loop():
    """WKV7 oracle against the per-token update written over whole [B, H] batches:
    S <- S diag(d) + (S a) b^T + v k^T with d = exp(-e^-0.5 sigmoid(w)), y = S r."""
    torch.manual_seed(2)
    B, T, H, N = 3, 6, 2, 4
    r, w, k, v, a, b = (torch.randn(B, T, H, N, dtype=torch.float64) for _ in range(6))
    s0 = torch.randn(B, H, N, N, dtype=torch.float64)
    y, end = reference(r, w, k, v, a, b, s0)
    S = s0.clone()
    for t in range(T):
        d = torch.exp(-torch.exp(torch.tensor(-0.5, dtype=torch.float64)) * torch.sigmoid(w[:, t]))
        Sa = torch.einsum("bhij,bhj->bhi", S, a[:, t])
        S = S * d[:, :, None, :] + Sa[..., None] * b[:, t, :, None, :] + v[:, t, ..., None] * k[:, t, :, None, :]
        want = torch.einsum("bhij,bhj->bhi", S, r[:, t])
        torch.testing.assert_close(y[:, t].double(), want, rtol=1e-5, atol=1e-5)  # the oracle runs in fp32
    torch.testing.assert_close(end.double(), S, rtol=1e-5, atol=1e-5)
