"""Gated DeltaNet block on CUDA: the four input projections as one tcgen05 GEMM
(qkv | z | a | b), conv1d+SiLU with carried window, chunked delta rule, gated
RMSNorm, output projection."""
import torch

from . import f32, native
from .gemm import linear


def fused_weight(module, names, attr):
    """One [sum of outputs, in] bf16 weight for projections that read the same input, built once per module.
    bf16 parameters are re-pointed to views of it (the frozen teacher keeps a single copy of its weights)."""
    linears = [getattr(module, n) for n in names]
    w = getattr(module, attr, None)
    if w is not None and w.device == linears[0].weight.device:
        return w
    w = torch.cat([lin.weight.detach().to(torch.bfloat16) for lin in linears], 0).contiguous()
    o = 0
    for lin in linears:
        n = lin.weight.shape[0]
        if lin.weight.dtype == torch.bfloat16 and not lin.weight.requires_grad:
            lin.weight.data = w[o:o + n]
        o += n
    setattr(module, attr, w)
    return w


def gdn_forward(module, x, conv_state, rec_state):
    cfg = module.cfg
    B, T, C = x.shape
    Hk, Hv, D = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim
    x2 = x.reshape(B * T, C)
    # qkv, z, a and b in one GEMM; the consumers read column slices of its rows
    proj = linear(x2, fused_weight(module, ("in_proj_qkv", "in_proj_z", "in_proj_a", "in_proj_b"), "_in_weight"))
    nqkv, nz = module.in_proj_qkv.weight.shape[0], module.in_proj_z.weight.shape[0]
    qkv = proj[:, :nqkv].view(B, T, nqkv)
    z = proj[:, nqkv:nqkv + nz]
    ab = proj[:, nqkv + nz:]
    qkv, conv_state = native().conv1d_silu(qkv, conv_state.contiguous(), f32(module.conv1d.weight))
    rec_state = rec_state.contiguous()
    core = native().gdn_forward(qkv, ab[:, :Hv], ab[:, Hv:], f32(module.A_log), f32(module.dt_bias), rec_state, Hk, Hv, D)
    core = native().gated_rmsnorm(core, z, f32(module.norm.weight), module.norm.eps)
    return linear(core.view(B * T, Hv * D), module.out_proj.weight).view(B, T, C), conv_state, rec_state
