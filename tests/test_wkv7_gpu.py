"""Chunked WKV7 CUDA kernels against the fp32 autograd recurrence (nonzero s0)."""
import pytest
import torch

from rwkv_theseus_b200.ops.wkv7 import reference, wkv7

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


def _inputs(B, T, H, N, dtype, scale=.5):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T * 10 + N)
    xs = [torch.randn(B, T, H, N, device="cuda", generator=g) * scale for _ in range(6)]
    xs[1] = xs[1] * 4  # decay logits over a wide range
    kk = torch.nn.functional.normalize(torch.randn(B, T, H, N, device="cuda", generator=g), dim=-1)
    xs[4], xs[5] = -kk, kk * torch.rand(B, T, H, 1, device="cuda", generator=g)   # RWKV7 ICL form
    xs = [x.to(dtype).requires_grad_() for x in xs]
    s0 = (torch.randn(B, H, N, N, device="cuda", generator=g) * .1).requires_grad_()
    return xs, s0


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,N", [(2, 7, 2, 8), (2, 7, 2, 64), (1, 37, 3, 64), (2, 16, 1, 128), (2, 70, 3, 32),
                                     (1, 50, 2, 40), (1, 1, 2, 64), (3, 100, 2, 16)])
def test_forward_backward_match_autograd(dtype, B, T, H, N):
    xs, s0 = _inputs(B, T, H, N, dtype)
    ref_x = [x.detach().clone().requires_grad_() for x in xs]
    ref_s = s0.detach().clone().requires_grad_()
    y, state = wkv7(*xs, s0)
    yr, sr = reference(*ref_x, ref_s)
    bf = dtype == torch.bfloat16
    torch.testing.assert_close(y, yr, atol=2e-3 if bf else 2e-5, rtol=2e-2 if bf else 1e-4)
    torch.testing.assert_close(state, sr, atol=3e-5, rtol=3e-4)
    dy, ds = torch.randn_like(y), torch.randn_like(state)
    torch.autograd.backward((y, state), (dy, ds))
    torch.autograd.backward((yr, sr), (dy, ds))
    for a, b in zip([*xs, s0], [*ref_x, ref_s]):
        torch.testing.assert_close(a.grad, b.grad, atol=4e-3 if bf else 3e-5, rtol=2.5e-2 if bf else 5e-4)


@cuda
def test_backward_is_deterministic_and_chunking_invariant():
    xs, s0 = _inputs(2, 70, 2, 64, torch.float32)
    outs = []
    for _ in range(2):
        for x in [*xs, s0]:
            x.grad = None
        y, st = wkv7(*xs, s0)
        (y.square().sum() + st.sum()).backward()
        outs.append([x.grad.clone() for x in [*xs, s0]])
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    with torch.no_grad():
        full, end = wkv7(*xs, s0)
        a, mid = wkv7(*[x[:, :33] for x in xs], s0)
        b, end2 = wkv7(*[x[:, 33:] for x in xs], mid)
    torch.testing.assert_close(torch.cat([a, b], 1), full, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(end2, end, atol=1e-5, rtol=1e-4)


@cuda
def test_runs_on_current_stream():
    xs, s0 = _inputs(2, 40, 2, 64, torch.bfloat16)
    with torch.no_grad():
        expected, _ = wkv7(*xs, s0)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            actual, _ = wkv7(*xs, s0)
        torch.cuda.current_stream().wait_stream(stream)
    assert torch.equal(actual, expected)


@cuda
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,N", [(8, 1, 4, 64), (2, 3, 2, 32), (3, 4, 2, 128), (1, 1, 80, 64)])
def test_decode_step_kernel_matches_reference(dtype, B, T, H, N):
    """Inference calls of 1-4 tokens (no checkpoints) use the token-by-token kernel."""
    xs, s0 = _inputs(B, T, H, N, dtype)
    xs = [x.detach() for x in xs]
    with torch.no_grad():
        y, state = wkv7(*xs, s0.detach())
        yr, sr = reference(*xs, s0.detach())
    bf = dtype == torch.bfloat16
    torch.testing.assert_close(y, yr, atol=2e-3 if bf else 2e-5, rtol=2e-2 if bf else 1e-4)
    torch.testing.assert_close(state, sr, atol=3e-5, rtol=3e-4)
