"""Frozen Qwen3.5-family hybrid teacher (Gated DeltaNet + gated full attention).

An own implementation of the text model (no HF forward on any path): module
and parameter names mirror the HF checkpoint layout
(``model.layers.{i}.linear_attn.in_proj_qkv.weight`` ...) so HF
``save_pretrained`` directories load directly and exports stay HF-loadable.
The block math follows HF ``modeling_qwen3_5.py`` (decoder layer HF:744-783,
GDN HF:422-533, attention HF:647-692, MLP HF:695-708); ``ops.teacher``
dispatches each op to a CUDA kernel for CUDA tensors and to
``ops.reference`` on CPU.

State across chunks (``HybridCache``) holds, per layer, either the KV cache of
a full-attention block (preallocated to capacity, grown geometrically) or the
conv window and fp32 delta-rule state of a GDN block, plus a position cursor.
"""
from dataclasses import dataclass, field
import json
import math
from pathlib import Path

import torch
from torch import nn

from ..ops import teacher as T

_TEXT_FIELDS = ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                "num_attention_heads", "num_key_value_heads", "head_dim", "linear_num_key_heads",
                "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim",
                "linear_conv_kernel_dim")


@dataclass
class HybridConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    layer_types: list
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    partial_rotary_factor: float = 0.25
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    hidden_act: str = "silu"
    raw: dict = field(default_factory=dict, repr=False)

    @classmethod
    def from_dict(cls, data):
        text = data.get("text_config", data)
        if text.get("model_type", "qwen3_5_text") not in ("qwen3_5_text", "qwen3_5"):
            raise ValueError(f"Expected qwen3_5_text, got {text.get('model_type')}")
        values = {name: int(text[name]) for name in _TEXT_FIELDS}
        layer_types = text.get("layer_types")
        if layer_types is None:
            interval = int(text.get("full_attention_interval", 4))
            layer_types = ["full_attention" if (i + 1) % interval == 0 else "linear_attention"
                           for i in range(values["num_hidden_layers"])]
        rope = text.get("rope_parameters") or {}
        theta = rope.get("rope_theta", text.get("rope_theta", 10000.0))
        partial = rope.get("partial_rotary_factor", text.get("partial_rotary_factor", 0.25))
        if text.get("hidden_act", "silu") not in ("silu", "swish"):
            raise ValueError("Only SiLU/SwiGLU teachers are supported")
        if text.get("attention_bias", False):
            raise ValueError("Attention bias is not supported by this teacher implementation")
        return cls(**values, layer_types=list(layer_types), rms_norm_eps=float(text.get("rms_norm_eps", 1e-6)),
                   rope_theta=float(theta), partial_rotary_factor=float(partial),
                   tie_word_embeddings=bool(text.get("tie_word_embeddings", data.get("tie_word_embeddings", False))),
                   raw=dict(text))

    @classmethod
    def from_pretrained(cls, path):
        return cls.from_dict(json.loads((Path(path) / "config.json").read_text()))

    def to_dict(self):
        out = dict(self.raw)
        out.update({name: getattr(self, name) for name in _TEXT_FIELDS})
        out.update(model_type="qwen3_5_text", layer_types=list(self.layer_types), rms_norm_eps=self.rms_norm_eps,
                   tie_word_embeddings=self.tie_word_embeddings, attention_bias=False, hidden_act="silu")
        rope = dict(out.get("rope_parameters") or {})
        rope.update(rope_theta=self.rope_theta, partial_rotary_factor=self.partial_rotary_factor)
        rope.setdefault("rope_type", "default")
        out["rope_parameters"] = rope
        out.setdefault("architectures", ["Qwen3_5ForCausalLM"])
        return out

    @property
    def rotary_dim(self):
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def conv_dim(self):
        return 2 * self.linear_num_key_heads * self.linear_key_head_dim + \
            self.linear_num_value_heads * self.linear_value_head_dim


def _linear(fan_in, fan_out):
    return nn.Linear(fan_in, fan_out, bias=False)


class RMSNorm(nn.Module):
    """Qwen RMSNorm with (1 + weight) scaling; weight initialised at zero."""

    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(dim))
        self.eps = eps

    def forward(self, x):
        return T.rmsnorm(x, self.weight, self.eps)


class GatedRMSNorm(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps


class MLP(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.gate_proj = _linear(cfg.hidden_size, cfg.intermediate_size)
        self.up_proj = _linear(cfg.hidden_size, cfg.intermediate_size)
        self.down_proj = _linear(cfg.intermediate_size, cfg.hidden_size)

    def forward(self, x):
        return T.swiglu_mlp(x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight)


class Conv1dWeight(nn.Module):
    """Holds ``conv1d.weight`` [C, 1, K] under the HF name (no bias)."""

    def __init__(self, channels, kernel):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(channels, 1, kernel))
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))


class GatedDeltaNet(nn.Module):
    def __init__(self, cfg, layer_idx):
        super().__init__()
        self.cfg, self.layer_idx = cfg, layer_idx
        key_dim = cfg.linear_num_key_heads * cfg.linear_key_head_dim
        value_dim = cfg.linear_num_value_heads * cfg.linear_value_head_dim
        self.key_dim, self.value_dim = key_dim, value_dim
        self.conv1d = Conv1dWeight(cfg.conv_dim, cfg.linear_conv_kernel_dim)
        self.dt_bias = nn.Parameter(torch.ones(cfg.linear_num_value_heads))
        self.A_log = nn.Parameter(torch.empty(cfg.linear_num_value_heads).uniform_(0, 16).log_())
        self.norm = GatedRMSNorm(cfg.linear_value_head_dim, cfg.rms_norm_eps)
        self.out_proj = _linear(value_dim, cfg.hidden_size)
        self.in_proj_qkv = _linear(cfg.hidden_size, cfg.conv_dim)
        self.in_proj_z = _linear(cfg.hidden_size, value_dim)
        self.in_proj_b = _linear(cfg.hidden_size, cfg.linear_num_value_heads)
        self.in_proj_a = _linear(cfg.hidden_size, cfg.linear_num_value_heads)

    def forward(self, x, cache=None):
        state = cache.layers[self.layer_idx] if cache is not None else None
        return T.gated_deltanet(self, x, state)


class Attention(nn.Module):
    def __init__(self, cfg, layer_idx):
        super().__init__()
        self.cfg, self.layer_idx = cfg, layer_idx
        q_out = cfg.num_attention_heads * cfg.head_dim
        kv_out = cfg.num_key_value_heads * cfg.head_dim
        self.q_proj = _linear(cfg.hidden_size, 2 * q_out)
        self.k_proj = _linear(cfg.hidden_size, kv_out)
        self.v_proj = _linear(cfg.hidden_size, kv_out)
        self.o_proj = _linear(q_out, cfg.hidden_size)
        self.q_norm = RMSNorm(cfg.head_dim, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(cfg.head_dim, cfg.rms_norm_eps)

    def forward(self, hidden_states, rope=None, cache=None):
        state = cache.layers[self.layer_idx] if cache is not None else None
        return T.gated_attention(self, hidden_states, rope, state)


class DecoderLayer(nn.Module):
    def __init__(self, cfg, layer_idx):
        super().__init__()
        self.layer_type = cfg.layer_types[layer_idx]
        if self.layer_type == "linear_attention":
            self.linear_attn = GatedDeltaNet(cfg, layer_idx)
        elif self.layer_type == "full_attention":
            self.self_attn = Attention(cfg, layer_idx)
        else:
            raise ValueError(f"Unknown layer type {self.layer_type}")
        self.mlp = MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)

    def mixer(self, h, rope, cache):
        if self.layer_type == "linear_attention":
            return self.linear_attn(h, cache)
        out = self.self_attn(h, rope=rope, cache=cache)
        return out[0] if isinstance(out, tuple) else out

    def forward(self, x, rope, cache):
        h = self.mixer(self.input_layernorm(x), rope, cache)
        x, h = T.add_rmsnorm(x, h, self.post_attention_layernorm.weight, self.post_attention_layernorm.eps)
        return T.residual_add(x, self.mlp(h))


class TextModel(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(DecoderLayer(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        dim = cfg.rotary_dim
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    def forward(self, ids, positions, cache, stop_at=None):
        """``positions``: first absolute position (int) or a tensor of consecutive positions. With ``stop_at``
        the pass ends inside block ``stop_at`` and returns its mixer (attention) output: the blocks before it and
        its own mixer update the cache; its residual and MLP, the later blocks and the final norm are not run."""
        start = int(positions[0]) if torch.is_tensor(positions) else int(positions)
        x = T.embed(ids, self.embed_tokens.weight)
        rope = T.rope_tables(self.inv_freq, start, ids.shape[1], x.device, x.dtype)
        # Each block's MLP residual is added by the next norm's fused add + RMSNorm kernel (x + mlp rounded to
        # x.dtype, then normalised), the same values as DecoderLayer.forward followed by the next input norm.
        pending = None
        for index, layer in enumerate(self.layers):
            norm = layer.input_layernorm
            if pending is None:
                normed = norm(x)
            else:
                x, normed = T.add_rmsnorm(x, pending, norm.weight, norm.eps)
            h = layer.mixer(normed, rope, cache)
            if index == stop_at:
                return h
            x, h = T.add_rmsnorm(x, h, layer.post_attention_layernorm.weight, layer.post_attention_layernorm.eps)
            pending = layer.mlp(h)
        return T.add_rmsnorm(x, pending, self.norm.weight, self.norm.eps)[1]


class HybridForCausalLM(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.model = TextModel(cfg)
        self.lm_head = _linear(cfg.hidden_size, cfg.vocab_size)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight

    def init_weights(self, std=0.02, generator=None):
        """Random init in the HF scheme: N(0, std) linears/embedding, zero RMSNorm,
        unit gated-norm and dt_bias, log U(0,16) A_log."""
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("norm.weight") and "linear_attn" in name:
                    p.fill_(1.0)
                elif name.endswith("layernorm.weight") or name.endswith("q_norm.weight") or \
                        name.endswith("k_norm.weight") or name == "model.norm.weight":
                    p.zero_()
                elif name.endswith("dt_bias"):
                    p.fill_(1.0)
                elif name.endswith("A_log"):
                    p.copy_(torch.empty(p.shape, device=p.device).uniform_(0, 16, generator=generator).log_())
                elif name.endswith("conv1d.weight"):
                    p.normal_(0.0, std, generator=generator)
                else:
                    p.normal_(0.0, std, generator=generator)
        return self


class HybridCache:
    """Per-layer recurrent state and KV cache with an explicit position cursor."""

    def __init__(self, config):
        self.config = config
        self.cursor = 0
        self.layers = [dict(kind=kind) for kind in config.layer_types]

    def get_seq_length(self, layer_idx=0):
        return self.cursor

    def reset(self):
        """Start a new window: position 0, empty KV caches and zero recurrent states. The buffers are kept (their
        stale entries are never read: attention masks keys past the length, and a fresh recurrent state is
        cleared in place before its first use), so document starts allocate and copy nothing."""
        self.cursor = 0
        for layer in self.layers:
            if "keys" in layer:
                layer["length"] = 0
            if "recurrent" in layer:
                layer["fresh"] = True

    def state_dict(self):
        out = []
        for layer in self.layers:
            entry = {"kind": layer["kind"]}
            if layer["kind"] == "full_attention" and "keys" in layer:
                n = layer["length"]
                entry.update(keys=layer["keys"][:, :n].clone(), values=layer["values"][:, :n].clone(), length=n)
            elif layer["kind"] == "linear_attention" and "recurrent" in layer:
                entry.update(conv=layer["conv"].clone(), recurrent=layer["recurrent"].clone())
            out.append(entry)
        return out

    def load_state_dict(self, layers, device):
        if len(layers) != len(self.layers):
            raise ValueError("Cache layer count mismatch")
        for i, entry in enumerate(layers):
            fresh = {"kind": self.layers[i]["kind"]}
            if entry.get("kind", fresh["kind"]) != fresh["kind"]:
                raise ValueError("Cache layer kind mismatch")
            if "keys" in entry:
                fresh.update(keys=entry["keys"].to(device).contiguous(), values=entry["values"].to(device).contiguous(),
                             length=int(entry["length"]))
            if "recurrent" in entry:
                fresh.update(conv=entry["conv"].to(device), recurrent=entry["recurrent"].to(device))
            self.layers[i] = fresh
