"""GEMM operators on the tcgen05 kernel (bf16 operands, fp32 accumulation in TMEM).

``matmul(a, b, a_t, b_t)`` computes ``op(a) @ op(b)^T`` where ``op`` is the
identity or a transpose of a row-major operand; transposed operands are read
directly as MN-major tiles by TMA (no transpose copy). Used for every
projection of the teacher and the students (forward, input gradients and
weight gradients).
"""
import torch

from . import native


def _2d(x):
    return x.reshape(-1, x.shape[-1])


def linear(x, weight):
    """y = x @ weight^T (weight [out, in]); bf16 result."""
    w = weight if weight.dtype == torch.bfloat16 else weight.to(torch.bfloat16)
    x2 = _2d(x)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = native().gemm(x2, False, w, False, 0, 1.0, None)
    return out.view(*x.shape[:-1], weight.shape[0])


def linear_f32(x, weight):
    out = native().gemm(_2d(x), False, weight, False, 1, 1.0, None)
    return out.view(*x.shape[:-1], weight.shape[0])


def input_grad(dy, weight):
    """dx = dy @ weight (weight [out, in] read MN-major); bf16 result."""
    out = native().gemm(_2d(dy), False, weight, True, 0, 1.0, None)
    return out.view(*dy.shape[:-1], weight.shape[1])


def weight_grad_(grad, dy, x, alpha=1.0):
    """grad[out, in] += alpha * dy^T @ x (fp32 accumulate; dy, x bf16 row-major [tokens, .])."""
    native().gemm(_2d(dy), True, _2d(x), True, 2, float(alpha), grad)
    return grad


def swiglu(x, w_gate, w_up):
    """silu(x @ w_gate^T) * (x @ w_up^T), one dual-operand GEMM."""
    out = native().gemm_swiglu(_2d(x), w_gate, w_up)
    return out.view(*x.shape[:-1], w_gate.shape[0])
