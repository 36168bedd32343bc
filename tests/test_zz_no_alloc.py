"""The allocation-free GDN forward (rt_gdn_forward_noalloc), called through its exported C symbol.

Callers that cannot allocate device memory while running the layer (a fixed
memory pool, a decode loop that must not synchronise on cudaMalloc, a plain C
caller) use this entry point; its scratch is a static device array inside the
library. The test calls it with ctypes, twice in a row on a carried state,
and checks it against the allocating entry point within the tolerance of the
GDN kernel test. It is collected last and also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA unavailable")
CUDA_ERROR_INVALID_VALUE = 1


def _entry():
    from rwkv_theseus_b200.ops import native
    ext = native()
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.rt_gdn_forward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_long,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    cap = lib.rt_gdn_noalloc_capacity_floats
    cap.restype = ctypes.c_long
    return ext, fn, cap()


def _call(fn, qkv, ab, Hv, A_log, dt_bias, state, out, B, T, Hk, D):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(qkv.data_ptr(), qkv.size(2), ab[:, :Hv].data_ptr(), ab[:, Hv:].data_ptr(), ab.stride(0),
              A_log.data_ptr(), dt_bias.data_ptr(), state.data_ptr(), out.data_ptr(), B, T, Hk, Hv, D, stream)


@cuda
@pytest.mark.parametrize("B,T,Hk,Hv,D", [(2, 45, 2, 6, 64), (1, 33, 16, 48, 128)])
def test_noalloc_matches_allocating_entry_point(B, T, Hk, Hv, D):
    ext, fn, capacity = _entry()
    assert capacity == 1 << 20
    g = torch.Generator(device="cuda").manual_seed(7)
    A_log = torch.rand(Hv, device="cuda", generator=g) * 3
    dt_bias = torch.randn(Hv, device="cuda", generator=g)
    state0 = torch.randn(B, Hv, D, D, device="cuda", generator=g) * 0.1
    state_ref, state_new = state0.clone(), state0.clone()
    for call in range(2):  # two calls in a row, each continuing from the previous state
        qkv = (torch.randn(B, T, 2 * Hk * D + Hv * D, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        ab = torch.randn(B * T, 2 * Hv, device="cuda", generator=g).to(torch.bfloat16)
        expected = ext.gdn_forward(qkv, ab[:, :Hv], ab[:, Hv:], A_log, dt_bias, state_ref, Hk, Hv, D)
        out = torch.empty_like(expected)
        rc = _call(fn, qkv, ab, Hv, A_log, dt_bias, state_new, out, B, T, Hk, D)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: cudaError {rc}"
        torch.testing.assert_close(out.float(), expected.float(), atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(state_new, state_ref, atol=2e-3, rtol=2e-3)


@cuda
def test_noalloc_rejects_work_beyond_its_scratch():
    ext, fn, capacity = _entry()
    B, T, Hk, Hv, D = 1, 4096, 16, 48, 128
    qkv = torch.zeros(B, T, 2 * Hk * D + Hv * D, device="cuda", dtype=torch.bfloat16)
    ab = torch.zeros(B * T, 2 * Hv, device="cuda", dtype=torch.bfloat16)
    state = torch.zeros(B, Hv, D, D, device="cuda")
    out = torch.zeros(B, T, Hv, D, device="cuda", dtype=torch.bfloat16)
    A_log, dt_bias = torch.zeros(Hv, device="cuda"), torch.zeros(Hv, device="cuda")
    assert _call(fn, qkv, ab, Hv, A_log, dt_bias, state, out, B, T, Hk, D) == CUDA_ERROR_INVALID_VALUE
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(state) == 0


@cuda
@pytest.mark.parametrize("case", ["odd_row_stride", "short_row_stride", "short_ab_stride", "misaligned_qkv"])
def test_noalloc_rejects_strides_and_pointers_the_kernels_cannot_read(case):
    """Plain C callers pass raw strides and pointers; a layout the 16-byte row copies cannot read is refused
    before anything is launched (no output or state is written)."""
    ext, fn, _ = _entry()
    B, T, Hk, Hv, D = 1, 20, 2, 6, 64
    width = 2 * Hk * D + Hv * D
    qkv_buf = torch.zeros(B * T * (width + 16) + 64, device="cuda", dtype=torch.bfloat16)
    row_stride, ab_stride, offset = width, 2 * Hv, 0
    if case == "odd_row_stride":
        row_stride = width + 3
    elif case == "short_row_stride":
        row_stride = width - 8
    elif case == "short_ab_stride":
        ab_stride = Hv - 1
    else:
        offset = 1  # one bf16 past a 16-byte boundary
    ab = torch.zeros(B * T, 2 * Hv, device="cuda", dtype=torch.bfloat16)
    state = torch.zeros(B, Hv, D, D, device="cuda")
    out = torch.zeros(B, T, Hv, D, device="cuda", dtype=torch.bfloat16)
    A_log, dt_bias = torch.zeros(Hv, device="cuda"), torch.zeros(Hv, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(qkv_buf.data_ptr() + 2 * offset, row_stride, ab.data_ptr(), ab[:, Hv:].data_ptr(), ab_stride,
            A_log.data_ptr(), dt_bias.data_ptr(), state.data_ptr(), out.data_ptr(), B, T, Hk, Hv, D, stream)
    torch.cuda.synchronize()
    assert rc == CUDA_ERROR_INVALID_VALUE
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(state) == 0
