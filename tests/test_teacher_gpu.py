"""CUDA teacher path (own kernels) against the fp32 CPU reference of the same weights."""
import pytest
import torch

from rwkv_theseus_b200.models.hf_io import random_model
from rwkv_theseus_b200.models.qwen35 import HybridCache, HybridConfig
from rwkv_theseus_b200.ops import native, reference as R

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


def cfg(D=64):
    return HybridConfig(vocab_size=300, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                        num_attention_heads=4, num_key_value_heads=2, head_dim=64, linear_num_key_heads=2,
                        linear_num_value_heads=4, linear_key_head_dim=D, linear_value_head_dim=D,
                        linear_conv_kernel_dim=4, layer_types=["linear_attention", "full_attention"] * 2,
                        rope_theta=1e6, partial_rotary_factor=0.25)


@cuda
@pytest.mark.parametrize("D", [64, 128])
def test_chunked_forward_matches_fp32_reference(D):
    torch.manual_seed(0)
    c = cfg(D)
    model = random_model(c, "cuda")
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or name.endswith("_norm.weight"):
                p.normal_(0, 0.1)
    ref = random_model(c, "cpu", dtype=torch.float32)
    ref.load_state_dict({k: v.float().cpu() for k, v in model.state_dict().items()})
    ids = torch.randint(0, c.vocab_size, (2, 70))
    with torch.no_grad():
        expected = ref.model(ids, 0, HybridCache(ref.config))
        cache, parts = HybridCache(model.config), []
        for a, b in [(0, 33), (33, 34), (34, 70)]:
            parts.append(model.model(ids[:, a:b].cuda(), a, cache))
            cache.cursor = b
        got = torch.cat(parts, 1).float().cpu()
    err = (got - expected).abs().max().item()
    assert err < 0.05 * expected.abs().max().item(), err


@cuda
@pytest.mark.parametrize("B,T,Hk,Hv,D", [(2, 45, 2, 6, 64),       # serial 16-step path
                                         (2, 200, 2, 6, 64),      # WY path, partial last chunk
                                         (1, 128, 2, 4, 128),     # WY path, exact chunks
                                         (1, 333, 4, 12, 128)])   # WY path, 6 chunks, GQA 3
def test_gdn_kernel_matches_reference_recurrence(B, T, Hk, Hv, D):
    torch.manual_seed(1)
    qkv = (torch.randn(B, T, 2 * Hk * D + Hv * D, device="cuda") * 0.5).to(torch.bfloat16)
    ab = (torch.randn(B * T, 2 * Hv, device="cuda")).to(torch.bfloat16)
    A_log = torch.rand(Hv, device="cuda") * 3
    dt_bias = torch.randn(Hv, device="cuda")
    state = torch.randn(B, Hv, D, D, device="cuda") * 0.1
    ref_state = state.clone()
    out = native().gdn_forward(qkv, ab[:, :Hv], ab[:, Hv:], A_log, dt_bias, state, Hk, Hv, D)
    q, k, v = torch.split(qkv.float(), [Hk * D, Hk * D, Hv * D], -1)
    a, b = ab[:, :Hv].float().view(B, T, Hv), ab[:, Hv:].view(B, T, Hv)
    g = -A_log.exp() * torch.nn.functional.softplus(a + dt_bias)
    beta = torch.sigmoid(b).float()
    ro, rs = R.gated_delta_rule(q.view(B, T, Hk, D), k.view(B, T, Hk, D), v.view(B, T, Hv, D), g, beta, ref_state)
    torch.testing.assert_close(out.float(), ro.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(state, rs, atol=2e-3, rtol=2e-3)


@cuda
@pytest.mark.parametrize("T,C", [(17, 512),     # vectorised paths, one conv segment
                                 (70, 5120),    # 27B width: 5 words per thread, three conv segments
                                 (2, 512),      # fewer steps than the conv window (state carried through)
                                 (9, 516)])     # width not a multiple of 8: scalar paths
def test_norm_conv_ops(T, C):
    torch.manual_seed(2)
    x = torch.randn(3, T, C, device="cuda").to(torch.bfloat16)
    h = torch.randn_like(x)
    w = torch.randn(C, device="cuda") * 0.1
    torch.testing.assert_close(native().rmsnorm_1p(x, w, 1e-6).float(), R.rmsnorm_1p(x.float(), w, 1e-6),
                               atol=3e-2, rtol=2e-2)
    s, n = native().add_rmsnorm_1p(x, h, w, 1e-6)
    torch.testing.assert_close(s, x + h)
    torch.testing.assert_close(n.float(), R.rmsnorm_1p((x + h).float(), w, 1e-6), atol=3e-2, rtol=2e-2)
    state = torch.randn(3, 3, C, device="cuda").to(torch.bfloat16)
    cw = torch.randn(C, 1, 4, device="cuda") * 0.3
    y, ns = native().conv1d_silu(x, state, cw)
    ry, rns = R.causal_conv1d_silu(x.float(), state.float(), cw[:, 0].float())
    torch.testing.assert_close(y.float(), ry, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(ns.float(), rns)
    z = torch.randn(51, 128, device="cuda").to(torch.bfloat16)
    xx = torch.randn(51, 128, device="cuda").to(torch.bfloat16)
    gw = torch.rand(128, device="cuda")
    torch.testing.assert_close(native().gated_rmsnorm(xx, z, gw, 1e-6).float(),
                               R.gated_rmsnorm(xx.float(), z.float(), gw, 1e-6), atol=3e-2, rtol=3e-2)


@cuda
def test_smoke_step():
    from rwkv_theseus_b200.smoke import run_smoke
    reports = run_smoke(torch.device("cuda", 0))
    assert reports.shape == (2, 5)


@cuda
@pytest.mark.parametrize("B", [1, 2])
def test_gdn_state_carry_across_mixed_call_lengths(B):
    """Calls of 512, 257, 511, 1, 383, 17 and 63 tokens (both kernel paths, decode-sized steps) carry the
    recurrent state exactly like one pass of the reference recurrence."""
    torch.manual_seed(3)
    Hk, Hv, D = 2, 4, 128
    lengths = [512, 257, 511, 1, 383, 17, 63]
    T = sum(lengths)
    qkv = (torch.randn(B, T, 2 * Hk * D + Hv * D, device="cuda") * 0.5).to(torch.bfloat16)
    ab = torch.randn(B, T, 2 * Hv, device="cuda").to(torch.bfloat16)
    A_log = torch.rand(Hv, device="cuda") * 2
    dt_bias = torch.randn(Hv, device="cuda")
    state = torch.zeros(B, Hv, D, D, device="cuda")
    outs, t0 = [], 0
    for n in lengths:
        piece = qkv[:, t0:t0 + n].contiguous()
        gates = ab[:, t0:t0 + n].reshape(B * n, 2 * Hv)
        outs.append(native().gdn_forward(piece, gates[:, :Hv], gates[:, Hv:], A_log, dt_bias, state, Hk, Hv, D))
        t0 += n
    out = torch.cat(outs, 1)
    q, k, v = torch.split(qkv.float(), [Hk * D, Hk * D, Hv * D], -1)
    a, b = ab[..., :Hv].float(), ab[..., Hv:]
    g = -A_log.exp() * torch.nn.functional.softplus(a + dt_bias)
    beta = torch.sigmoid(b).float()
    ro, rs = R.gated_delta_rule(q.view(B, T, Hk, D), k.view(B, T, Hk, D), v.view(B, T, Hv, D), g, beta,
                                torch.zeros(B, Hv, D, D, device="cuda"))
    torch.testing.assert_close(out.float(), ro.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(state, rs, atol=3e-3, rtol=3e-3)
