"""RWKV7 TimeMix student: the module that replaces one full-attention block.

Attribution: the TimeMix formulas (token-shift lerps, decay / in-context
learning-rate / gate LoRAs, the RWKV7 state update, per-head GroupNorm and
bonus term) and the initialisation schedule follow RWKV7 ``RWKV_Tmix_x070``
and ``generate_init_weight`` of RWKV-LM (BlinkDL; RWKV-Vibe/RWKV-LM-V7,
commit 665472dab30952de9379a3a3a01eaa3453f1ad4e, ``src/model.py``), licensed
under the Apache License 2.0 (see ``NOTICE`` at the project root). This file
restates them in its own code; it adds no v_first path between layers.

Parameter schema (23 tensors, names/shapes/order as reference
``theseus/timemix.py:29-59``)::

    x_r x_w x_k x_v x_a x_g   [1,1,C]   token-shift lerp coefficients
    w1 [C,R] w2 [R,C]                   decay LoRA (R = lora rank)
    a1 [C,R] a2 [R,C]                   in-context learning-rate LoRA
    w0 a0 [1,1,C]                       LoRA biases
    g1 [C,Rg] g2 [Rg,C]                 output-gate LoRA
    k_k k_a [1,1,C]   r_k [H,N]
    receptance/key/value/output.weight [C,C]
    ln_x.weight ln_x.bias [C]           per-head GroupNorm (eps 64e-5)

The initialisation schedule is the RWKV7 one (depth-dependent lerp
coefficients, zig-zag decay/ICL biases, orthogonal LoRA up-projections,
zero output projection) with ranks ``max(32, round(2.5 sqrt(C)/32)*32)`` and
``max(32, round(5 sqrt(C)/32)*32)``; both can be overridden.

``forward`` here is the PyTorch definition (CPU path and oracle; on CUDA its
WKV call uses the chunked kernel). Training on CUDA goes through
``models.student_fused`` which runs the same math as fused sm_100a kernels with
a hand-written backward.
"""
import math

import torch
from torch import nn
from torch.nn import functional as F

from ..ops.wkv7 import wkv7

PARAM_ORDER = ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g", "w1", "w2", "a1", "a2", "w0", "a0",
               "g1", "g2", "k_k", "k_a", "r_k", "receptance.weight", "key.weight", "value.weight",
               "output.weight", "ln_x.weight", "ln_x.bias")
GROUPNORM_EPS = 64e-5


def lora_ranks(width, lora_rank=None, gate_lora_rank=None):
    rank = lora_rank or max(32, round(2.5 * math.sqrt(width) / 32) * 32)
    gate = gate_lora_rank or max(32, round(5 * math.sqrt(width) / 32) * 32)
    return rank, gate


class TimeMix(nn.Module):
    def __init__(self, width, layer_idx, depth, head_size=64, backend="cuda", lora_rank=None,
                 gate_lora_rank=None):
        super().__init__()
        if width % head_size or head_size < 2:
            raise ValueError("width must be divisible by head_size >= 2")
        self.width, self.head_size = width, head_size
        self.heads, self.backend = width // head_size, backend
        self.layer_idx, self.depth = layer_idx, depth
        c, n = width, head_size
        rank, gate_rank = lora_ranks(width, lora_rank, gate_lora_rank)
        self.rank, self.gate_rank = rank, gate_rank
        ratio = layer_idx / max(depth - 1, 1)
        reverse = 1 - layer_idx / depth
        pos = torch.arange(c).reshape(1, 1, c) / c
        for name, power in (("r", .2), ("w", .9), ("k", .7), ("v", .7), ("a", .9), ("g", .2)):
            setattr(self, "x_" + name, nn.Parameter(1 - pos.pow(power * reverse)))
        ramp = torch.arange(c) / (c - 1) - .5
        zigzag = (torch.arange(c) % n - (n - 1) / 2) / ((n - 1) / 2)
        zigzag = zigzag * zigzag.abs()
        decay_bias = -6 + 6 * (torch.arange(c) / (c - 1)).pow(1 + ratio ** .3)
        for name in ("w", "a"):
            setattr(self, name + "1", nn.Parameter(torch.zeros(c, rank)))
            up = nn.Parameter(torch.empty(rank, c))
            nn.init.orthogonal_(up, gain=.1 * max(1, math.sqrt(rank / c)))
            setattr(self, name + "2", up)
        self.w0 = nn.Parameter((decay_bias + .5 + zigzag * 2.5).reshape(1, 1, c))
        self.a0 = nn.Parameter((-.19 + zigzag * .3 + ramp * .4).reshape(1, 1, c))
        self.g1 = nn.Parameter(torch.zeros(c, gate_rank))  # sigmoid(0) = 0.5: gate starts open
        self.g2 = nn.Parameter(torch.empty(gate_rank, c))
        nn.init.orthogonal_(self.g2, gain=.1 * max(1, math.sqrt(gate_rank / c)))
        self.k_k = nn.Parameter((.71 - ramp * .1).reshape(1, 1, c))
        self.k_a = nn.Parameter(torch.full((1, 1, c), 1.02))
        self.r_k = nn.Parameter(torch.full((self.heads, n), -.04))
        for name, gain in (("receptance", 1.), ("key", .1), ("value", 1.), ("output", 0.)):
            linear = nn.Linear(c, c, bias=False)
            if gain:
                nn.init.orthogonal_(linear.weight, gain=gain)
            else:
                nn.init.zeros_(linear.weight)
            setattr(self, name, linear)
        self.ln_x = nn.GroupNorm(self.heads, c, eps=GROUPNORM_EPS)
        nn.init.constant_(self.ln_x.weight, ((1 + layer_idx) / depth) ** .7)

    def initial_state(self, x):
        return {"shift": torch.zeros(x.shape[0], self.width, device=x.device, dtype=x.dtype),
                "wkv": torch.zeros(x.shape[0], self.heads, self.head_size, self.head_size,
                                   device=x.device, dtype=torch.float32)}

    def forward(self, x, state=None):
        if state is None:
            state = self.initial_state(x)
        batch, length, _ = x.shape
        delta = torch.cat([state["shift"].unsqueeze(1), x[:, :-1]], 1) - x
        mixed = {name: (x + delta * getattr(self, "x_" + name)).to(x.dtype) for name in "rwkvag"}
        r = self.receptance(mixed["r"])
        w = self.w0 + torch.tanh(mixed["w"] @ self.w1) @ self.w2
        k, v = self.key(mixed["k"]), self.value(mixed["v"])
        a = torch.sigmoid(self.a0 + (mixed["a"] @ self.a1) @ self.a2)
        g = torch.sigmoid(mixed["g"] @ self.g1) @ self.g2
        shape = (batch, length, self.heads, self.head_size)
        kk = F.normalize((k.float() * self.k_k).reshape(shape), dim=-1, eps=1e-12)
        k = k * (1 + (a - 1) * self.k_a)
        args = [z.reshape(shape).to(r.dtype).contiguous()
                for z in (r, w, k, v, -kk, kk * a.reshape(shape))]
        y, end = wkv7(*args, state["wkv"], backend=self.backend)
        with torch.autocast(x.device.type, enabled=False):
            y = F.group_norm(y.float().reshape(batch * length, self.width), self.heads,
                             self.ln_x.weight.float(), self.ln_x.bias.float(),
                             GROUPNORM_EPS).reshape(batch, length, self.width)
            bonus = ((r.float().reshape(shape) * k.float().reshape(shape) * self.r_k).sum(-1, keepdim=True)
                     * v.float().reshape(shape)).reshape(batch, length, self.width)
            y = ((y + bonus) * g.float()).to(x.dtype)
        return self.output(y).to(x.dtype), {"shift": x[:, -1], "wkv": end}


def detach_state(state):
    return None if state is None else {k: v.detach() for k, v in state.items()}
