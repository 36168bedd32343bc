"""The chunked WY form of the WKV7 forward (ops.wkv7_chunked) against the per-token recurrence, on CPU in fp64."""
import pytest
import torch

from rwkv_theseus_b200.ops.wkv7 import LOG_DECAY_SCALE, reference
from rwkv_theseus_b200.ops.wkv7_chunked import wkv7_chunked


def _recurrence64(r, w, k, v, a, b, s0):
    """The per-token recurrence of ops.wkv7.reference, kept in float64."""
    d = torch.exp(-LOG_DECAY_SCALE * torch.sigmoid(w))
    s, out = s0.clone(), []
    for t in range(r.shape[1]):
        sa = (s * a[:, t, :, None, :]).sum(-1)
        s = s * d[:, t, :, None, :] + sa[..., None] * b[:, t, :, None, :] + v[:, t, :, :, None] * k[:, t, :, None, :]
        out.append((s * r[:, t, :, None, :]).sum(-1))
    return torch.stack(out, 1), s


def _inputs(B, T, H, N, seed, w_shift=0.0):
    g = torch.Generator().manual_seed(seed)
    rnd = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    r, k, v = rnd(B, T, H, N), rnd(B, T, H, N), rnd(B, T, H, N)
    w = rnd(B, T, H, N) + w_shift
    kk = torch.nn.functional.normalize(rnd(B, T, H, N), dim=-1)       # RWKV7 in-context form: a = -kk, b = kk * gate
    a, b = -kk, kk * torch.sigmoid(rnd(B, T, H, N))
    s0 = rnd(B, H, N, N) * 0.1
    return r, w, k, v, a, b, s0


@pytest.mark.parametrize("T,chunk", [(150, 64), (64, 64), (37, 16), (200, 32)])
def test_chunked_matches_recurrence(T, chunk):
    xs = _inputs(2, T, 2, 16, seed=T + chunk)
    y_ref, s_ref = _recurrence64(*xs)
    y, s = wkv7_chunked(*xs, chunk=chunk)
    torch.testing.assert_close(y, y_ref, rtol=1e-9, atol=1e-9)
    torch.testing.assert_close(s, s_ref, rtol=1e-9, atol=1e-9)
    y32, _ = reference(*xs)  # the library's fp32 oracle agrees to fp32 rounding
    torch.testing.assert_close(y32.double(), y_ref, rtol=1e-3, atol=1e-4)


def test_strongest_decay_over_a_64_step_chunk_stays_in_fp32_range():
    """sigmoid(w) -> 1 everywhere: Lambda falls by e^{-1/2} per step, so e^{-Lambda} reaches about 7e16 at the end
    of a 64-step chunk. The chunk form still matches in fp64 and produces finite values in fp32."""
    xs = _inputs(1, 128, 1, 16, seed=3, w_shift=30.0)
    y_ref, s_ref = _recurrence64(*xs)
    y, s = wkv7_chunked(*xs, chunk=64)
    torch.testing.assert_close(y, y_ref, rtol=1e-8, atol=1e-9)
    torch.testing.assert_close(s, s_ref, rtol=1e-8, atol=1e-9)
    y32, s32 = wkv7_chunked(*xs, chunk=64, dtype=torch.float32)
    assert torch.isfinite(y32).all() and torch.isfinite(s32).all()
    torch.testing.assert_close(y32.double(), y_ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("T,chunk", [(150, 64), (37, 16), (64, 64)])
def test_chunked_backward_matches_autograd_of_the_recurrence(T, chunk):
    from rwkv_theseus_b200.ops.wkv7_chunked import wkv7_chunked_backward
    xs = [x.clone().requires_grad_(True) for x in _inputs(2, T, 2, 16, seed=7 * T + chunk)]
    y, s = _recurrence64(*xs)
    g = torch.Generator().manual_seed(11)
    dy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    ds = torch.randn(s.shape, generator=g, dtype=torch.float64)
    ref = torch.autograd.grad((y * dy).sum() + (s * ds).sum(), xs)
    got = wkv7_chunked_backward(*[x.detach() for x in xs], dy, ds, chunk=chunk)
    for name, g_got, g_ref in zip(("r", "w", "k", "v", "a", "b", "state"), got, ref):
        torch.testing.assert_close(g_got, g_ref, rtol=1e-8, atol=1e-9, msg=name)
