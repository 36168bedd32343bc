"""tcgen05 flash attention (head_dim 256, GQA, cache offset, fused gate) against an fp32 reference."""
import pytest
import torch

from rwkv_theseus_b200.ops import native

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


def reference(q, keys, values, gate, offset):
    B, T, Hq, D = q.shape
    L = offset + T
    k = keys[:, :L].float().repeat_interleave(Hq // keys.shape[2], 2)
    v = values[:, :L].float().repeat_interleave(Hq // keys.shape[2], 2)
    s = torch.einsum("bthd,blhd->bhtl", q.float(), k) / 16.0
    pos = torch.arange(T, device=q.device)[:, None] + offset
    s = s.masked_fill(torch.arange(L, device=q.device)[None] > pos, float("-inf"))
    o = torch.einsum("bhtl,blhd->bthd", torch.softmax(s, -1), v)
    return o * torch.sigmoid(gate.float())


@cuda
@pytest.mark.parametrize("B,T,Hq,Hkv,offset,cap", [(1, 128, 2, 1, 0, 256), (2, 70, 6, 1, 33, 128),
                                                    (1, 300, 4, 2, 500, 1024), (1, 1, 6, 1, 77, 80),
                                                    (1, 1024, 24, 4, 2048, 4096)])
def test_flash_attention_matches_reference(B, T, Hq, Hkv, offset, cap):
    g = torch.Generator(device="cuda").manual_seed(offset + T)
    D = 256
    q = torch.randn(B, T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    keys = torch.zeros(B, cap, Hkv, D, device="cuda", dtype=torch.bfloat16)
    values = torch.zeros_like(keys)
    keys[:, :offset + T] = (torch.randn(B, offset + T, Hkv, D, device="cuda", generator=g) * 2).to(torch.bfloat16)
    values[:, :offset + T] = torch.randn(B, offset + T, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    qg = torch.randn(B * T, Hq * 2 * D, device="cuda", generator=g).to(torch.bfloat16)
    gate = qg.view(B, T, Hq, 2 * D)[..., D:]
    out = native().flash_attention(q, keys, values, qg, offset)
    ref = reference(q, keys, values, gate, offset)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
