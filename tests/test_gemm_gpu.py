"""tcgen05 GEMM against an fp32 PyTorch matmul of the same bf16 operands."""
import pytest
import torch

from rwkv_theseus_b200.ops import native

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")


def _bf(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * 0.5).to(torch.bfloat16)


def _check(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, (err, scale)


@cuda
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 512), (1024, 5120, 5120), (37, 48, 5120),
                                   (1, 192, 5120), (130, 352, 192), (1000, 200, 352), (64, 64, 8)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
def test_layouts_and_tails(M, N, K, a_t, b_t):
    if (a_t and M % 8) or (b_t and N % 8):
        pytest.skip("MN-major operands need a row stride that is a multiple of 8")
    A = _bf(K, M, seed=1) if a_t else _bf(M, K, seed=1)
    B = _bf(K, N, seed=2) if b_t else _bf(N, K, seed=2)
    ref = (A.float().t() if a_t else A.float()) @ (B.float() if b_t else B.float().t())
    out = native().gemm(A, a_t, B, b_t, 0, 1.0, None)
    _check(out, ref)
    out32 = native().gemm(A, a_t, B, b_t, 1, 1.0, None)
    _check(out32, ref, 1e-3)


@cuda
def test_accumulate_epilogue():
    dy, x = _bf(300, 256, seed=3), _bf(300, 192, seed=4)
    grad = torch.randn(256, 192, device="cuda")
    expected = grad + 0.5 * dy.float().t() @ x.float()
    native().gemm(dy, True, x, True, 2, 0.5, grad)
    _check(grad, expected, 1e-3)


@cuda
def test_swiglu_epilogue():
    x, wg, wu = _bf(257, 512, seed=5), _bf(384, 512, seed=6), _bf(384, 512, seed=7)
    ref = torch.nn.functional.silu(x.float() @ wg.float().t()) * (x.float() @ wu.float().t())
    _check(native().gemm_swiglu(x, wg, wu), ref)


@cuda
def test_strided_rows_and_current_stream():
    big = _bf(512, 1024, seed=8)
    A = big[:, 256:768]                 # row stride 1024, unit inner stride
    B = _bf(640, 512, seed=9)
    ref = A.float() @ B.float().t()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        out = native().gemm(A, False, B, False, 0, 1.0, None)
    torch.cuda.current_stream().wait_stream(stream)
    _check(out, ref)


@pytest.mark.parametrize("M,N,K", [(1, 5120, 5120), (8, 10240, 5120), (8, 5120, 17408), (32, 384, 200),
                                   (5, 130, 72)])
def test_skinny_decode_gemm_matches_fp32(M, N, K):
    """M <= 32: split-K weight streaming path (swapped tiles, fp32 atomics), plain and SwiGLU."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA unavailable")
    from rwkv_theseus_b200.ops import native
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    u = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    got = native().gemm(x, False, w, False, 0, 1.0, None)
    torch.testing.assert_close(got.float(), ref, atol=2e-2, rtol=2e-2)
    sw = native().gemm_swiglu(x, w, u)
    ref_sw = torch.nn.functional.silu(ref) * (x.float() @ u.float().t())
    torch.testing.assert_close(sw.float(), ref_sw, atol=2e-2, rtol=2e-2)


SK = 1 << 16


@cuda
@pytest.mark.parametrize("M,N,K,bn", [(1024, 5120, 5120, 256),   # 160 tiles on 148 SMs: tiles split over 2 CTAs
                                      (256, 512, 5120, 256),     # 4 tiles of 80 k-blocks: ~37 CTAs per tile
                                      (300, 1000, 1000, 192),    # ragged M, N and K tails
                                      (1024, 5120, 17408, 224)])
def test_stream_k_matches_fp32(M, N, K, bn):
    A, B = _bf(M, K, seed=5), _bf(N, K, seed=6)
    ref = A.float() @ B.float().t()
    for rep in range(2):  # the second launch checks that the tile counters were left at zero
        out = native().gemm(A, False, B, False, 0, 1.0, None, bn | SK)
        _check(out, ref)
    out32 = native().gemm(A, False, B, False, 1, 1.0, None, bn | SK)
    _check(out32, ref, 1e-3)
    whole = native().gemm(A, False, B, False, 1, 1.0, None, bn)
    assert (out32 - whole).abs().max().item() <= 1e-4 * ref.abs().max().item()


@cuda
def test_stream_k_accumulate_mn_major():
    dy, x = _bf(1024, 640, seed=7), _bf(1024, 5120, seed=8)  # dW = dy^T x: 5 x 20 tiles, 16 k-blocks
    acc = torch.randn(640, 5120, device="cuda")
    ref = acc + 0.5 * (dy.float().t() @ x.float())
    native().gemm(dy, True, x, True, 2, 0.5, acc, 256 | SK)
    _check(acc, ref, 1e-3)


@cuda
@pytest.mark.parametrize("M,N,K,tuned", [(1024, 5120, 5120, True), (300, 1000, 1000, False), (37, 256, 512, False)])
def test_fused_loss_epilogue_matches_fp32(M, N, K, tuned):
    """Output GEMM with the NMSE/cosine loss in its epilogue vs the fp32 statistics and their gradient."""
    from rwkv_theseus_b200.losses import statistics
    x, w = _bf(M, K, seed=11), _bf(N, K, seed=12)
    target = (_bf(M, N, seed=13).float() * 3).to(torch.bfloat16)
    if tuned:  # a measured (possibly stream-K) tile choice for this shape bucket
        native().gemm(x, False, w, False, 0, 1.0, None)
    p = x.float() @ w.float().t()
    eps = 1e-6
    ref = statistics(p, target.float(), eps)
    denom = target.float().square().mean(-1, keepdim=True).clamp_min(eps)
    ref_grad = 2 * (p - target.float()) / (N * denom)
    stats = torch.zeros(3, device="cuda")
    dpred = native().gemm_nmse(x, w, target, stats, eps)
    torch.testing.assert_close(stats, ref, rtol=1e-3, atol=1e-3)
    _check(dpred, ref_grad)
    stats2 = torch.zeros(3, device="cuda")
    dpred2 = native().gemm_nmse(x, w, target, stats2, eps)
    assert torch.equal(dpred, dpred2)
    torch.testing.assert_close(stats2, stats, rtol=1e-5, atol=0)  # row sums gather tiles with float atomics


SP = 20  # tile choice bits 20..27: parallel split-K factor


@cuda
@pytest.mark.parametrize("M,N,K,tile", [(1024, 192, 5120, 64 | 16 << SP),    # LoRA down: 16 tiles x 9 parts
                                        (1024, 352, 5120, 128 | 8 << SP),    # 24 tiles x 6 parts (clamped)
                                        (300, 96, 1000, 64 | 12 << SP),      # ragged M, N, K
                                        (1024, 1024, 5120, 256 | 4 << SP)])
def test_parallel_split_k_matches_fp32(M, N, K, tile):
    A, B = _bf(M, K, seed=21), _bf(N, K, seed=22)
    ref = A.float() @ B.float().t()
    for rep in range(2):  # the second launch checks that the tile counters were reset
        _check(native().gemm(A, False, B, False, 0, 1.0, None, tile), ref)
    _check(native().gemm(A, False, B, False, 1, 1.0, None, tile), ref, 1e-3)
    dy, x = _bf(1024, 192, seed=23), _bf(1024, 640, seed=24)   # weight-gradient form, accumulate epilogue
    acc = torch.randn(192, 640, device="cuda")
    want = acc + 0.5 * (dy.float().t() @ x.float())
    native().gemm(dy, True, x, True, 2, 0.5, acc, 64 | 8 << SP)
    _check(acc, want, 1e-3)


# Fixed schedules for the grouped launch: whole tiles of 256 / 128 / 64 columns, stream-K, parallel split-K (S = 4).
# At 384 x 640 x 1216 every one of them runs as named for G = 2 and 3 (stream-K: at least one k-block per SM;
# split-K: tiles x S within the SM count).
M2 = 1 << 17  # tile choice bit: 256-row tiles (two M = 128 MMAs per k-step on one B tile)
_GROUP_SCHEDULES = [256, 128, 64, 256 | (1 << 16), 128 | (1 << 16), 256 | (4 << 20),
                    256 | M2, 128 | M2, 256 | M2 | (1 << 16), 128 | M2 | (1 << 16)]


@cuda
@pytest.mark.parametrize("G", [2, 3])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("tile", [0] + _GROUP_SCHEDULES)
def test_grouped_gemm_matches_fp32(G, a_t, b_t, tile):
    """G problems of one shape in one launch (shared tile numbering and stream-K space) equal G fp32 matmuls."""
    M, N, K = 384, 640, 1216
    As = [_bf(K, M, seed=10 + g) if a_t else _bf(M, K, seed=10 + g) for g in range(G)]
    Bs = [_bf(K, N, seed=20 + g) if b_t else _bf(N, K, seed=20 + g) for g in range(G)]
    refs = [(A.float().t() if a_t else A.float()) @ (B.float() if b_t else B.float().t()) for A, B in zip(As, Bs)]
    outs = native().gemm_group(As, a_t, Bs, b_t, 0, 1.0, [], tile)
    for out, ref in zip(outs, refs):
        _check(out, ref)
    # fp32 store, then accumulate alpha * result into the given outputs (the weight-gradient epilogues)
    f32 = native().gemm_group(As, a_t, Bs, b_t, 1, 1.0, [], tile)
    for out, ref in zip(f32, refs):
        _check(out, ref, 1e-3)
    base = [torch.randn(M, N, device="cuda") for _ in range(G)]
    acc = [b.clone() for b in base]
    native().gemm_group(As, a_t, Bs, b_t, 2, 0.5, acc, tile)
    for out, b, ref in zip(acc, base, refs):
        _check(out, b + 0.5 * ref, 1e-3)


@cuda
def test_grouped_gemm_student_shape_and_strided_outputs():
    """The r/k/v shape of the 27B student (1024 x 5120 x 5120, three problems) writing into slices of one buffer,
    as the fused student writes its input gradients into the mix-gradient tensor."""
    M, N, K = 1024, 5120, 5120
    As = [_bf(M, K, seed=30 + g) for g in range(3)]
    Bs = [_bf(N, K, seed=40 + g) for g in range(3)]
    dst = torch.zeros(6, M, N, device="cuda", dtype=torch.bfloat16)
    outs = [dst.select(0, i) for i in (0, 2, 3)]
    native().gemm_group(As, False, Bs, False, 0, 1.0, outs, 0)
    for i, (A, B) in zip((0, 2, 3), zip(As, Bs)):
        _check(dst[i], A.float() @ B.float().t())
    for i in (1, 4, 5):
        assert dst[i].abs().max().item() == 0.0


def test_grouped_gemm_rejects_mismatched_problems():
    if not torch.cuda.is_available():
        pytest.skip("CUDA unavailable")
    A, B = _bf(128, 64, seed=1), _bf(64, 64, seed=2)
    with pytest.raises(RuntimeError):
        native().gemm_group([A, _bf(128, 128, seed=3)], False, [B, B], False, 0, 1.0, [], 0)
    with pytest.raises(RuntimeError):
        native().gemm_group([A] * 4, False, [B] * 4, False, 0, 1.0, [], 0)


@cuda
@pytest.mark.parametrize("M,N,K", [(1024, 5120, 1024), (296, 384, 704), (1000, 200, 352), (256, 64, 64)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("tile", [256 | M2, 128 | M2, 256 | M2 | (1 << 16), 128 | M2 | (1 << 16)])
def test_256_row_tiles_match_fp32(M, N, K, a_t, b_t, tile):
    """256-row tiles: partial row and column tiles, all operand layouts, store / fp32 / accumulate epilogues, whole
    tiles and stream-K (run twice: the stream-K counters must be left at zero)."""
    if (a_t and M % 8) or (b_t and N % 8):
        pytest.skip("MN-major operands need a row stride that is a multiple of 8")
    A = _bf(K, M, seed=51) if a_t else _bf(M, K, seed=51)
    B = _bf(K, N, seed=52) if b_t else _bf(N, K, seed=52)
    ref = (A.float().t() if a_t else A.float()) @ (B.float() if b_t else B.float().t())
    for _ in range(2):
        _check(native().gemm(A, a_t, B, b_t, 0, 1.0, None, tile), ref)
    _check(native().gemm(A, a_t, B, b_t, 1, 1.0, None, tile), ref, 1e-3)
    base = torch.randn(M, N, device="cuda")
    acc = base.clone()
    native().gemm(A, a_t, B, b_t, 2, -0.5, acc, tile)
    _check(acc, base - 0.5 * ref, 1e-3)


@cuda
@pytest.mark.parametrize("M,N,K", [(1024, 1536, 1024), (300, 384, 512)])
@pytest.mark.parametrize("tile", [0, 128, 128 | M2])
def test_swiglu_tile_rows(M, N, K, tile):
    """SwiGLU with 128- and 256-row tiles (and the measured choice) against fp32."""
    x, wg, wu = _bf(M, K, seed=61), _bf(N, K, seed=62), _bf(N, K, seed=63)
    ref = torch.nn.functional.silu(x.float() @ wg.float().t()) * (x.float() @ wu.float().t())
    _check(native().gemm_swiglu(x, wg, wu, tile), ref)
