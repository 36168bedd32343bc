"""One-GPU robustness checks: a bounded device wait that runs out records a status instead of hanging
(the peer flag is never set), and kernels that promise determinism give bitwise-identical results on
repeated runs."""
import pytest
import torch

from rwkv_theseus_b200.ops import native

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


@cuda
@pytest.mark.parametrize("mode", [1, 0])  # three-kernel path; fused update/pull kernel
def test_exchange_wait_for_absent_peer_times_out_with_status(mode):
    ext = native()
    n, dev = 1024, torch.device("cuda", 0)
    mine = {k: torch.zeros(n, device=dev) for k in ("g", "p", "m", "v")}
    ghost = {k: torch.zeros(n, device=dev) for k in ("g", "p")}  # "rank 1": local buffers nobody updates
    shadow = [torch.zeros(n, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    sig = [torch.zeros(ext.exchange_signal_words(), dtype=torch.int32, device=dev) for _ in range(2)]
    stats, report = torch.tensor([1.0, 1.0, 4.0], device=dev), torch.zeros(5, device=dev)
    ext.exchange_update([mine["g"].data_ptr(), ghost["g"].data_ptr()], [mine["p"].data_ptr(), ghost["p"].data_ptr()],
                        [shadow[0].data_ptr(), shadow[1].data_ptr()], [sig[0].data_ptr(), sig[1].data_ptr()],
                        0, 2, n, mine["m"], mine["v"], stats, report, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1.0, 1, n,
                        1, 0.3, 4, mode)
    torch.cuda.synchronize()  # returns after the three bounded waits (about 1 s), the context stays usable
    words = sig[0][24:28].cpu().tolist()
    assert words[0] == 1 and words[3] == 1  # status "gradients ready" missing from rank 1
    assert not mine["p"].any()  # nothing was applied
    assert int(sig[1][0].item()) == 1  # our own arrival was published to the peer's flags
    torch.ones(1, device=dev).add_(1)  # the device still runs work


@cuda
def test_wkv7_backward_is_bitwise_deterministic():
    from rwkv_theseus_b200.ops.wkv7 import wkv7
    g = torch.Generator(device="cuda").manual_seed(5)
    B, T, H, N = 2, 70, 4, 64
    xs = [(torch.randn(B, T, H, N, device="cuda", generator=g) * 0.5).to(torch.bfloat16) for _ in range(6)]
    s0 = torch.randn(B, H, N, N, device="cuda", generator=g) * 0.1
    grads = []
    for _ in range(2):
        leaves = [x.detach().clone().requires_grad_() for x in xs] + [s0.clone().requires_grad_()]
        y, end = wkv7(*leaves)
        (y.float().square().sum() + end.square().sum()).backward()
        grads.append([t.grad.clone() for t in leaves])
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@cuda
def test_gdn_forward_is_bitwise_deterministic():
    g = torch.Generator(device="cuda").manual_seed(6)
    Hk, Hv, D, T = 2, 6, 128, 300
    qkv = (torch.randn(1, T, 2 * Hk * D + Hv * D, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    ab = torch.randn(T, 2 * Hv, device="cuda", generator=g).to(torch.bfloat16)
    A_log, dt = torch.rand(Hv, device="cuda", generator=g), torch.randn(Hv, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        state = torch.zeros(1, Hv, D, D, device="cuda")
        out = native().gdn_forward(qkv, ab[:, :Hv], ab[:, Hv:], A_log, dt, state, Hk, Hv, D)
        outs.append((out, state))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
