"""Gated full-attention block on CUDA.

Projections run on the tcgen05 GEMM; q/k per-head RMSNorm(1+w) and partial
RoPE are one kernel that writes q into a fresh buffer and k (with v) straight
into the preallocated KV cache at the chunk's positions; the output gate
sigmoid(g) multiplies the attention output before ``o_proj``.
"""
import torch
from torch.nn import functional as F

from . import f32, native
from .gdn import fused_weight
from .gemm import linear


def _ensure_cache(state, B, T, Hkv, D, device):
    """Grow the [B, cap, Hkv, D] KV cache to hold T more tokens; return the current length."""
    keys = state.get("keys")
    length = state.get("length", 0) if keys is not None and keys.shape[0] == B else 0
    if keys is not None and keys.shape[0] != B:
        keys = None
    need = length + T
    if keys is None or keys.shape[1] < need:
        cap = max(need, 2 * (keys.shape[1] if keys is not None else 0), 1024)
        # Zero-filled: attention tiles read whole key blocks, and masked keys must hold finite values. The cache
        # outlives window resets (the length restarts at 0), so it grows only until it holds the longest window.
        new_k = torch.empty(B, cap, Hkv, D, device=device, dtype=torch.bfloat16)
        new_v = torch.empty_like(new_k)
        native().zero_(new_k)
        native().zero_(new_v)
        if keys is not None and length:
            new_k[:, :length].copy_(keys[:, :length])
            new_v[:, :length].copy_(state["values"][:, :length])
        state["keys"], state["values"] = new_k, new_v
    return length


def core_attention(q, k_all, v_all, offset):
    """Causal GQA attention for head sizes the tcgen05 kernel does not cover (PyTorch SDPA)."""
    B, T, Hq, D = q.shape
    L = k_all.shape[1]
    rows = torch.arange(T, device=q.device)[:, None] + offset
    mask = torch.arange(L, device=q.device)[None] <= rows
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k_all.transpose(1, 2), v_all.transpose(1, 2),
                                         attn_mask=mask, scale=D ** -0.5, enable_gqa=True)
    return out.transpose(1, 2)


def attention_block(module, x, rope, state):
    cfg = module.cfg
    B, T, C = x.shape
    Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    inv_freq, pos0 = rope[2], rope[3]
    rot = cfg.rotary_dim
    x2 = x.reshape(B * T, C)
    proj = linear(x2, fused_weight(module, ("q_proj", "k_proj", "v_proj"), "_qkv_weight"))  # one GEMM: q|g, k, v
    nq, nk = module.q_proj.weight.shape[0], module.k_proj.weight.shape[0]
    qg = proj[:, :nq]                                       # [BT, Hq * 2D]: per head [q | gate]
    k = proj[:, nq:nq + nk]
    v = proj[:, nq + nk:]
    q = torch.empty(B, T, Hq, D, device=x.device, dtype=torch.bfloat16)
    native().norm_rope_(qg, Hq, f32(module.q_norm.weight), f32(inv_freq), q, pos0, 0, rot, module.q_norm.eps)
    if state is None:
        state = {}
    length = _ensure_cache(state, B, T, Hkv, D, x.device)
    native().norm_rope_(k, Hkv, f32(module.k_norm.weight), f32(inv_freq), state["keys"], pos0, length, rot,
                        module.k_norm.eps)
    native().copy_rows_(v, state["values"], length)
    state["length"] = length + T
    if D == 256:
        out = native().flash_attention(q, state["keys"], state["values"], qg, length).view(B * T, Hq * D)
    else:
        out = core_attention(q, state["keys"][:, :length + T], state["values"][:, :length + T], length)
        gate = qg.view(B, T, Hq, 2 * D)[..., D:]
        out = (out * torch.sigmoid(gate)).reshape(B * T, Hq * D)
    return linear(out, module.o_proj.weight).view(B, T, C)
