"""Teacher-block operators: CUDA tensors run the sm_100a kernels of the
extension, CPU tensors run ``ops.reference``.

Each function is the unit the teacher's modules call; the CUDA versions fuse
what the HF implementation runs as separate ATen kernels (norm + residual,
conv + SiLU + state carry, q/k norm + RoPE + attention + output gate,
SwiGLU gate/up + activation).
"""
import torch
from torch.nn import functional as F

from . import reference as R
from . import f32, native


def _cuda(x):
    return x.is_cuda


def linear(x, weight):
    """y = x @ weight^T in the activation dtype (bf16 on the CUDA path)."""
    if _cuda(x):
        from .gemm import linear as gemm_linear
        return gemm_linear(x, weight)
    return F.linear(x, weight.to(x.dtype))


def embed(ids, weight):
    """Embedding lookup; CUDA bf16 tables use this package's row-gather kernel."""
    if ids.is_cuda and weight.dtype == torch.bfloat16 and weight.is_contiguous() and weight.shape[1] % 8 == 0:
        return native().embed_rows(ids, weight)
    return F.embedding(ids, weight)


def rmsnorm(x, weight, eps):
    if _cuda(x):
        return native().rmsnorm_1p(x.contiguous(), f32(weight), float(eps))
    return R.rmsnorm_1p(x, weight, eps)


def add_rmsnorm(x, h, weight, eps):
    """(x + h, rmsnorm(x + h)) with the sum rounded to x.dtype first (as HF does)."""
    if _cuda(x):
        return tuple(native().add_rmsnorm_1p(x.contiguous(), h.contiguous(), f32(weight), float(eps)))
    s = x + h
    return s, R.rmsnorm_1p(s, weight, eps)


def residual_add(x, y):
    return x + y


def rope_tables(inv_freq, start, length, device, dtype):
    """(cos, sin, inv_freq, start) for positions start..start+length-1; on CUDA the
    kernels compute the angles themselves and cos/sin are not materialised."""
    if device.type == "cuda":
        return None, None, inv_freq, start
    positions = torch.arange(start, start + length, device=device)
    cos, sin = R.rope_tables(inv_freq, positions, dtype)
    return cos, sin, inv_freq, start


def swiglu_mlp(x, w_gate, w_up, w_down):
    if _cuda(x):
        from .gemm import swiglu, linear as gemm_linear
        return gemm_linear(swiglu(x, w_gate, w_up), w_down)
    return linear(F.silu(linear(x, w_gate)) * linear(x, w_up), w_down)


def _gdn_state(module, state, B, device, dtype):
    """(conv window, recurrent state) of the layer: the carried ones, or zeros at a window start (a kept buffer
    cleared in place by this package's kernel when the cache was reset)."""
    cfg = module.cfg
    K = cfg.linear_conv_kernel_dim
    if state is not None and "recurrent" in state and state["recurrent"].shape[0] == B:
        if state.pop("fresh", False):
            if device.type == "cuda":
                native().zero_(state["conv"])
                native().zero_(state["recurrent"])
            else:
                state["conv"].zero_()
                state["recurrent"].zero_()
        return state["conv"], state["recurrent"]
    conv = torch.zeros(B, K - 1, cfg.conv_dim, device=device, dtype=dtype)
    rec = torch.zeros(B, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim,
                      device=device, dtype=torch.float32)
    return conv, rec


def gated_deltanet(module, x, state):
    cfg = module.cfg
    B, T, _ = x.shape
    Hk, Dk = cfg.linear_num_key_heads, cfg.linear_key_head_dim
    Hv, Dv = cfg.linear_num_value_heads, cfg.linear_value_head_dim
    conv, rec = _gdn_state(module, state, B, x.device, x.dtype)
    if _cuda(x):
        from .gdn import gdn_forward
        out, conv, rec = gdn_forward(module, x, conv, rec)
    else:
        qkv = linear(x, module.in_proj_qkv.weight)
        z = linear(x, module.in_proj_z.weight)
        b = linear(x, module.in_proj_b.weight)
        a = linear(x, module.in_proj_a.weight)
        qkv, conv = R.causal_conv1d_silu(qkv, conv, module.conv1d.weight[:, 0, :])
        q, k, v = torch.split(qkv, [module.key_dim, module.key_dim, module.value_dim], -1)
        q = q.reshape(B, T, Hk, Dk)
        k = k.reshape(B, T, Hk, Dk)
        v = v.reshape(B, T, Hv, Dv)
        beta = torch.sigmoid(b)
        g = -module.A_log.float().exp() * F.softplus(a.float() + module.dt_bias.float())
        core, rec = R.gated_delta_rule(q, k, v, g, beta, rec)
        core = R.gated_rmsnorm(core.reshape(-1, Dv), z.reshape(-1, Dv), module.norm.weight,
                               module.norm.eps).reshape(B, T, Hv * Dv)
        out = linear(core, module.out_proj.weight)
    if state is not None:
        state["conv"], state["recurrent"] = conv, rec
    return out


def _append_kv(state, k, v):
    """Append [B,T,H,D] keys/values to a capacity-doubling cache; return full views."""
    B, T = k.shape[:2]
    length = state.get("length", 0)
    keys = state.get("keys")
    if keys is None or keys.shape[0] != B:
        length, keys = 0, None
    need = length + T
    if keys is None or keys.shape[1] < need:
        cap = max(need, 2 * (keys.shape[1] if keys is not None else 0), 256)
        new_k = torch.empty(B, cap, *k.shape[2:], device=k.device, dtype=k.dtype)
        new_v = torch.empty_like(new_k)
        if keys is not None and length:
            new_k[:, :length] = keys[:, :length]
            new_v[:, :length] = state["values"][:, :length]
        state["keys"], state["values"] = new_k, new_v
    state["keys"][:, length:need] = k
    state["values"][:, length:need] = v
    state["length"] = need
    return state["keys"][:, :need], state["values"][:, :need], length


def gated_attention(module, x, rope, state):
    cfg = module.cfg
    B, T, _ = x.shape
    Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    if _cuda(x):
        from .attention import attention_block
        return attention_block(module, x, rope, state)
    cos, sin = rope[0], rope[1]
    qg = linear(x, module.q_proj.weight).view(B, T, Hq, 2 * D)
    q, gate = qg[..., :D], qg[..., D:]
    gate = gate.reshape(B, T, Hq * D)
    q = R.rmsnorm_1p(q, module.q_norm.weight, module.q_norm.eps)
    k = R.rmsnorm_1p(linear(x, module.k_proj.weight).view(B, T, Hkv, D), module.k_norm.weight, module.k_norm.eps)
    v = linear(x, module.v_proj.weight).view(B, T, Hkv, D)
    q, k = R.apply_rope(q, cos, sin), R.apply_rope(k, cos, sin)
    if state is not None:
        k_all, v_all, offset = _append_kv(state, k, v)
    else:
        k_all, v_all, offset = k, v, 0
    out = R.attention(q, k_all, v_all, offset).reshape(B, T, Hq * D)
    out = out * torch.sigmoid(gate)
    return linear(out, module.o_proj.weight)
