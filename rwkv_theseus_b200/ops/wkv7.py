"""RWKV7 state recurrence (the DPLR "WKV7" operator).

Attribution: the recurrence (decay clamp, state update and readout) is the
RWKV7 one of RWKV-LM (BlinkDL; RWKV-Vibe/RWKV-LM-V7, commit
665472dab30952de9379a3a3a01eaa3453f1ad4e, ``cuda/rwkv7_clampw.cu``), Apache
License 2.0 (see ``NOTICE`` at the project root). The chunked kernels that
evaluate it here are this project's own.

State layout ``[batch, head, value i, key j]``. Per step (reference
``theseus/wkv7.py:16-28`` and ``kernels/wkv7_state.cu:12-40``)::

    d_t = exp(-e^{-1/2} * sigmoid(w_t))           (decay clamped to [0.545, 1))
    S_t = S_{t-1} diag(d_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T
    y_t = S_t r_t

The CUDA implementation is chunked (16 steps per chunk): inside a chunk the
low-rank term is solved with a unit-lower-triangular system, so work is
matrix-shaped and the serial dependency is one step per chunk instead of one
per token. Forward stores only the chunk-boundary states (not the full
per-token history the reference keeps, ``wkv7_state.cpp:21-22``) and backward
recomputes inside each chunk; no atomics are used, the value rows of a head are
split across a thread-block cluster and the key-side gradients are reduced
through distributed shared memory in a fixed order (deterministic).
"""
import torch

from . import native

LOG_DECAY_SCALE = 0.6065306597126334  # e^{-1/2}


def reference(r, w, k, v, a, b, state):
    """fp32 per-token recurrence; returns (y in the input dtype, final state fp32)."""
    dtype = r.dtype
    r, w, k, v, a, b = [x.float() for x in (r, w, k, v, a, b)]
    decay = torch.exp(-LOG_DECAY_SCALE * torch.sigmoid(w))
    s = state.float()
    out = []
    for t in range(r.shape[1]):
        sa = (s * a[:, t, :, None, :]).sum(-1)
        s = (s * decay[:, t, :, None, :] + sa[..., None] * b[:, t, :, None, :]
             + v[:, t, :, :, None] * k[:, t, :, None, :])
        out.append((s * r[:, t, :, None, :]).sum(-1))
    return torch.stack(out, 1).to(dtype), s


def _check(xs, s0):
    r = xs[0]
    if r.dim() != 4:
        raise ValueError("expected [B,T,H,N] inputs")
    B, T, H, N = r.shape
    if not 2 <= N <= 128:
        raise ValueError("head size must be in 2..128")
    for x in xs:
        if x.shape != r.shape or x.dtype != r.dtype or x.device != r.device:
            raise ValueError("WKV7 inputs must share shape, dtype and device")
    if s0.shape != (B, H, N, N):
        raise ValueError(f"state must be [B,H,N,N], got {tuple(s0.shape)}")


class _WKV7(torch.autograd.Function):
    @staticmethod
    def forward(ctx, r, w, k, v, a, b, s0):
        xs = [x.contiguous() for x in (r, w, k, v, a, b)]
        s0 = s0.float().contiguous()
        y, end, checkpoints, records = native().wkv7_forward(*xs, s0, True)
        ctx.save_for_backward(*xs, checkpoints, records)
        return y, end

    @staticmethod
    def backward(ctx, dy, dend):
        *xs, checkpoints, records = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(xs[0])
        if dend is None:
            dend = torch.zeros_like(checkpoints[:, :, 0])
        grads = native().wkv7_backward(*xs, checkpoints, records, dy.to(xs[0].dtype).contiguous(),
                                       dend.float().contiguous())
        return tuple(g.to(x.dtype) for g, x in zip(grads[:6], xs)) + (grads[6],)


def wkv7(r, w, k, v, a, b, state, backend="cuda"):
    """Differentiable WKV7; CPU tensors (or ``backend='reference'``) use the oracle."""
    if backend == "reference" or not r.is_cuda:
        if backend == "cuda" and not r.is_cuda:
            raise ValueError("CUDA backend requested on CPU; use backend='reference' for tests")
        return reference(r, w, k, v, a, b, state)
    if backend != "cuda":
        raise ValueError(f"Unknown WKV backend: {backend}")
    _check((r, w, k, v, a, b), state)
    needs_grad = torch.is_grad_enabled() and any(x.requires_grad for x in (r, w, k, v, a, b, state))
    if not needs_grad:
        xs = [x.contiguous() for x in (r, w, k, v, a, b)]
        y, end, _, _ = native().wkv7_forward(*xs, state.float().contiguous(), False)
        return y, end
    return _WKV7.apply(r, w, k, v, a, b, state)
