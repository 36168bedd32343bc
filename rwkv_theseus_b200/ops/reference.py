"""Plain PyTorch definitions of every teacher/student op.

These are the CPU execution path (Gloo tests, tiny fixtures) and the oracles
the CUDA kernels are tested against. They follow the math of the Qwen3.5
hybrid text model (HF ``modeling_qwen3_5.py``: RMSNorm with (1+w) at
HF:711-723, gated RMSNorm HF:175-190, causal conv1d HF:210-226, gated delta
rule HF:318-353, attention HF:647-692) with one deliberate difference: the
convolution and delta-rule state are always carried across chunks, which the
chunked HF 5.5 path does not do (it restarts both at every multi-token call).
"""
import torch
from torch.nn import functional as F


def rmsnorm_1p(x, weight, eps):
    """Qwen RMSNorm: normalise in fp32, scale by (1 + w), cast back to x.dtype."""
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (out * (1.0 + weight.float())).type_as(x)


def gated_rmsnorm(x, gate, weight, eps):
    """GDN output norm: w * norm(x) (in x.dtype) times SiLU(gate) in fp32."""
    dtype = x.dtype
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    out = weight * xf.to(dtype)
    out = out * F.silu(gate.float())
    return out.to(dtype)


def causal_conv1d_silu(x, state, weight):
    """Depthwise causal conv over time + SiLU with carried state.

    x: [B, T, C] (channels last), state: [B, K-1, C] previous inputs (oldest
    first), weight: [C, K] (tap K-1 multiplies the newest input).
    Returns (y [B, T, C] in x.dtype, new_state [B, K-1, C]).
    """
    K = weight.shape[-1]
    full = torch.cat([state.to(x.dtype), x], 1)
    taps = full.unfold(1, K, 1)  # [B, T, C, K]
    y = (taps.float() * weight.float()).sum(-1)
    new_state = full[:, full.shape[1] - (K - 1):]
    return F.silu(y).to(x.dtype), new_state.contiguous()


def l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gated_delta_rule(q, k, v, g, beta, state):
    """Recurrent gated delta rule with in-kernel q/k L2 norm and GQA.

    q, k: [B, T, Hk, Dk]; v: [B, T, Hv, Dv]; g (log decay), beta: [B, T, Hv];
    state: [B, Hv, Dk, Dv] fp32. Value head h reads key head h // (Hv / Hk).
    Returns (out [B, T, Hv, Dv] in v.dtype, new state fp32).
    """
    dtype = v.dtype
    rep = v.shape[2] // q.shape[2]
    q = l2norm(q.float()).repeat_interleave(rep, dim=2) * q.shape[-1] ** -0.5
    k = l2norm(k.float()).repeat_interleave(rep, dim=2)
    v, g, beta = v.float(), g.float(), beta.float()
    s = state.float()
    out = []
    for t in range(q.shape[1]):
        s = s * g[:, t, :, None, None].exp()
        mem = (s * k[:, t, :, :, None]).sum(-2)
        delta = (v[:, t] - mem) * beta[:, t, :, None]
        s = s + k[:, t, :, :, None] * delta[:, :, None, :]
        out.append((s * q[:, t, :, :, None]).sum(-2))
    return torch.stack(out, 1).to(dtype), s


def rope_tables(inv_freq, positions, dtype):
    freqs = positions.float()[:, None] * inv_freq.float()[None]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    """Partial rotary embedding on the first ``cos.shape[-1]`` dims. x: [B,T,H,D]."""
    rot = cos.shape[-1]
    xr, xp = x[..., :rot], x[..., rot:]
    half = rot // 2
    rotated = torch.cat([-xr[..., half:], xr[..., :half]], -1)
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat([xr * c + rotated * s, xp], -1)


def attention(q, k_all, v_all, offset):
    """Causal GQA attention of T queries against a cache of L >= T keys.

    q: [B, T, Hq, D]; k_all, v_all: [B, L, Hkv, D]; query t sits at absolute
    position offset + t and sees keys 0..offset+t. Returns [B, T, Hq, D].
    """
    B, T, Hq, D = q.shape
    L, Hkv = k_all.shape[1], k_all.shape[2]
    rep = Hq // Hkv
    qh = q.transpose(1, 2)
    kh = k_all.transpose(1, 2).repeat_interleave(rep, 1)
    vh = v_all.transpose(1, 2).repeat_interleave(rep, 1)
    rows = torch.arange(T, device=q.device)[:, None] + offset
    cols = torch.arange(L, device=q.device)[None]
    mask = cols <= rows
    out = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, scale=D ** -0.5)
    return out.transpose(1, 2)
