"""The tcgen05 WKV7 path (bf16, head size 64, at least 128 steps; chunks of 64) against the fp32 recurrence.

Its products take tf32 operands (fp32 accumulation, fp32 state), so it is compared with relative-norm bounds a
few times above the errors measured on a B200 (y about 1.7e-3 of its norm, final state about 2e-4, gradients
3e-4 to 1.5e-3), and with the chunk-16 CUDA-core path on the same inputs."""
import pytest
import torch

from rwkv_theseus_b200.ops import native
from rwkv_theseus_b200.ops.wkv7 import reference, wkv7

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


def inputs(B, T, H, seed, scale=.5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = [torch.randn(B, T, H, 64, device="cuda", generator=g) * scale for _ in range(6)]
    xs[1] = xs[1] * 4  # decay logits over a wide range
    kk = torch.nn.functional.normalize(torch.randn(B, T, H, 64, device="cuda", generator=g), dim=-1)
    xs[4], xs[5] = -kk, kk * torch.rand(B, T, H, 1, device="cuda", generator=g)
    xs = [x.to(torch.bfloat16).contiguous() for x in xs]
    s0 = torch.randn(B, H, 64, 64, device="cuda", generator=g) * .1
    return xs, s0


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@cuda
@pytest.mark.parametrize("B,T,H", [(1, 128, 2), (2, 200, 3), (1, 1024, 2), (3, 130, 1)])
def test_forward_and_gradients_match_the_fp32_recurrence(B, T, H):
    ext = native()
    xs, s0 = inputs(B, T, H, seed=B * 100 + T + H)
    y, end, ckpt, records = ext.wkv7_forward(*xs, s0, True)
    assert records.numel() > 0 and ckpt.shape == (B, H, (T + 63) // 64 + 1, 64, 64)
    ref_x = [x.float().requires_grad_() for x in xs]
    ref_s = s0.clone().requires_grad_()
    y_ref, end_ref = reference(*ref_x, ref_s)
    assert rel(y, y_ref) < 6e-3 and rel(end, end_ref) < 1e-3
    dy, dend = torch.randn_like(y_ref).to(torch.bfloat16), torch.randn_like(end_ref)
    grads = ext.wkv7_backward(*xs, ckpt, records, dy, dend)
    torch.autograd.backward((y_ref, end_ref), (dy.float(), dend))
    for name, got, want in zip("r w k v a b s0".split(), grads, [x.grad for x in ref_x] + [ref_s.grad]):
        assert rel(got, want) < 6e-3, name
    assert ext.wkv7_tc_fault() == 0


@cuda
def test_autograd_op_uses_the_tensor_core_path_and_agrees_with_chunk16():
    ext = native()
    xs, s0 = inputs(1, 256, 4, seed=5)
    leaves = [x.clone().requires_grad_() for x in xs]
    y, end = wkv7(*leaves, s0)
    (y.float().square().mean() + end.square().mean()).backward()
    tc_grads = [x.grad.clone() for x in leaves]
    ext.wkv7_tc_enable(False)
    try:
        leaves2 = [x.clone().requires_grad_() for x in xs]
        y2, end2 = wkv7(*leaves2, s0)
        (y2.float().square().mean() + end2.square().mean()).backward()
    finally:
        ext.wkv7_tc_enable(True)
    assert rel(y, y2) < 6e-3 and rel(end, end2) < 1e-3
    for a, b in zip(tc_grads, [x.grad for x in leaves2]):
        assert rel(a, b) < 8e-3


@cuda
def test_state_carry_across_calls_and_determinism():
    ext = native()
    xs, s0 = inputs(2, 384, 2, seed=9)
    with torch.no_grad():
        full, end = wkv7(*xs, s0)
        first, mid = wkv7(*[x[:, :192].contiguous() for x in xs], s0)
        second, end2 = wkv7(*[x[:, 192:].contiguous() for x in xs], mid)
    assert rel(torch.cat([first, second], 1), full) < 2e-3 and rel(end2, end) < 5e-4
    y, e, ckpt, records = ext.wkv7_forward(*xs, s0, True)
    dy, dend = torch.randn_like(y), torch.randn_like(e)
    g1 = ext.wkv7_backward(*xs, ckpt, records, dy, dend)
    g2 = ext.wkv7_backward(*xs, ckpt, records, dy, dend)
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))
