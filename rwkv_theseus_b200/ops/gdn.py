"""Gated DeltaNet block on CUDA: projections (tcgen05 GEMM), conv1d+SiLU with
carried window, chunked delta rule (two kernels: Gram/normalise prep and the
recurrent chunk pass), gated RMSNorm, output projection."""
import torch

from . import f32, native
from .gemm import linear


def _merged_ab(module):
    w = getattr(module, "_ab_weight", None)
    if w is None or w.device != module.in_proj_a.weight.device:
        w = torch.cat([module.in_proj_a.weight, module.in_proj_b.weight], 0).to(torch.bfloat16).contiguous()
        module._ab_weight = w
    return w


def gdn_forward(module, x, conv_state, rec_state):
    cfg = module.cfg
    B, T, C = x.shape
    Hk, Hv, D = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim
    x2 = x.reshape(B * T, C)
    qkv = linear(x2, module.in_proj_qkv.weight)
    z = linear(x2, module.in_proj_z.weight)
    ab = linear(x2, _merged_ab(module))
    qkv, conv_state = native().conv1d_silu(qkv.view(B, T, -1), conv_state.contiguous(), f32(module.conv1d.weight))
    rec_state = rec_state.contiguous()
    core = native().gdn_forward(qkv, ab[:, :Hv], ab[:, Hv:], f32(module.A_log), f32(module.dt_bias), rec_state, Hk, Hv, D)
    core = native().gated_rmsnorm(core, z, f32(module.norm.weight), module.norm.eps)
    return linear(core.view(B * T, Hv * D), module.out_proj.weight).view(B, T, C), conv_state, rec_state
