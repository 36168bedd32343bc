"""One-pass KL kernel and the lm_head logits path of validation against fp64 PyTorch."""
import pytest
import torch
from torch.nn import functional as F

from rwkv_theseus_b200.losses import kl_sum

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


def _kl64(s, t):
    ls, lt = F.log_softmax(s.double(), -1), F.log_softmax(t.double(), -1)
    return (lt.exp() * (lt - ls)).sum(-1)


@cuda
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,V", [(37, 1001), (3, 248077), (1, 7)])
def test_kl_rows_matches_fp64(dtype, rows, V):
    from rwkv_theseus_b200.ops import native
    g = torch.Generator(device="cuda").manual_seed(rows + V)
    s = (torch.randn(rows, V, device="cuda", generator=g) * 4).to(dtype)
    t = (s.float() + torch.randn(rows, V, device="cuda", generator=g)).to(dtype)
    got = native().kl_rows(s, t)
    ref = _kl64(s, t)
    torch.testing.assert_close(got.double(), ref, rtol=2e-4, atol=1e-5)
    torch.testing.assert_close(kl_sum(s.view(1, rows, V), t.view(1, rows, V)).double(), ref.sum(), rtol=2e-4,
                               atol=1e-4)


@cuda
def test_validation_logits_use_tcgen05_gemm():
    from rwkv_theseus_b200.validation import _logits
    g = torch.Generator(device="cuda").manual_seed(5)
    hidden = torch.randn(2, 16, 256, device="cuda", generator=g).to(torch.bfloat16)
    head = (torch.randn(1001, 256, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    got = _logits(hidden, head)
    ref = hidden.float() @ head.float().t()
    assert got.dtype == torch.bfloat16 and got.shape == (2, 16, 1001)
    torch.testing.assert_close(got.float(), ref, rtol=2e-2, atol=2e-2)
