"""HF-layout checkpoint IO for the hybrid teacher (safetensors, sharded).

Reads ``config.json`` + ``model.safetensors`` or
``model.safetensors.index.json`` shards (multimodal checkpoints with a
``model.language_model.`` prefix are remapped, ``model.visual.*`` and
``mtp.*`` tensors are ignored), and writes the same layout: shards of at most
``max_shard_bytes`` named ``model-XXXXX-of-YYYYY.safetensors`` with an index,
or a single ``model.safetensors``.
"""
import json
import os
from pathlib import Path

import torch
from safetensors import safe_open
from safetensors.torch import load_file, save_file

from .qwen35 import HybridConfig, HybridForCausalLM

_IGNORED = ("model.visual.", "mtp.")


def _canonical(key):
    if key.startswith("model.language_model."):
        return "model." + key[len("model.language_model."):]
    return key


def shard_files(path):
    path = Path(path)
    index = path / "model.safetensors.index.json"
    if index.exists():
        return sorted(set(json.loads(index.read_text())["weight_map"].values()))
    if (path / "model.safetensors").exists():
        return ["model.safetensors"]
    files = sorted(p.name for p in path.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"No safetensors checkpoint in {path}")
    return files


def weight_map(path):
    """Canonical tensor name -> shard file."""
    path = Path(path)
    mapping = {}
    for shard in shard_files(path):
        with safe_open(str(path / shard), framework="pt") as f:
            for key in f.keys():
                mapping[_canonical(key)] = (shard, key)
    return mapping


def build_empty(cfg, device="meta", dtype=torch.bfloat16):
    with torch.device(device):
        model = HybridForCausalLM(cfg)
    return model.to(dtype=dtype)


def load_model(path, device, dtype=torch.bfloat16):
    """Strict text-only loader: every model tensor present, nothing unexpected."""
    path = Path(path).resolve()
    cfg = HybridConfig.from_pretrained(path)
    model = build_empty(cfg, "meta", dtype)
    expected = set(model.state_dict())
    seen, unexpected = set(), []
    for shard in shard_files(path):
        tensors = load_file(str(path / shard), device=str(device))
        state = {}
        for key, value in tensors.items():
            name = _canonical(key)
            if name.startswith(_IGNORED):
                continue
            if name not in expected:
                unexpected.append(name)
                continue
            state[name] = value.to(dtype)
        model.load_state_dict(state, strict=False, assign=True)
        seen.update(state)
    if cfg.tie_word_embeddings and "lm_head.weight" not in seen:
        model.lm_head.weight = model.model.embed_tokens.weight
        seen.add("lm_head.weight")
    missing = expected - seen
    if missing or unexpected:
        raise RuntimeError(f"Text checkpoint mismatch: missing={sorted(missing)[:8]} unexpected={unexpected[:8]}")
    finalize(model, device)
    return model


def finalize(model, device):
    """Recreate non-persistent buffers on the target device and freeze."""
    cfg = model.config
    dim = cfg.rotary_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    model.model.inv_freq = inv_freq.to(device)
    model.requires_grad_(False).eval()
    return model


def random_model(cfg, device, dtype=torch.bfloat16, seed=0):
    """Random-init teacher materialised directly on ``device`` (no CPU copy)."""
    model = build_empty(cfg, "meta", dtype)
    model = model.to_empty(device=device)
    if cfg.tie_word_embeddings:
        model.lm_head.weight = model.model.embed_tokens.weight
    gen = torch.Generator(device=device).manual_seed(seed)
    model.init_weights(generator=gen)
    return finalize(model, device)


def save_model(model, path, max_shard_bytes=5 * 1024 ** 3, extra_state=None):
    """Write config.json and sharded safetensors in the HF layout."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    state = {k: v.detach().contiguous() for k, v in (extra_state or model.state_dict()).items()}
    if model.config.tie_word_embeddings:
        state.pop("lm_head.weight", None)
    shards, current, size = [], {}, 0
    for key in sorted(state):
        nbytes = state[key].numel() * state[key].element_size()
        if current and size + nbytes > max_shard_bytes:
            shards.append(current)
            current, size = {}, 0
        current[key] = state[key]
        size += nbytes
    if current or not shards:
        shards.append(current)
    config = model.config.to_dict()
    config["dtype"] = str(next(iter(state.values())).dtype).removeprefix("torch.") if state else "bfloat16"
    (path / "config.json").write_text(json.dumps(config, indent=2))
    if len(shards) == 1:
        save_file({k: v.cpu() for k, v in shards[0].items()}, str(path / "model.safetensors"),
                  metadata={"format": "pt"})
        return
    mapping, total = {}, 0
    for i, shard in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file({k: v.cpu() for k, v in shard.items()}, str(path / name), metadata={"format": "pt"})
        for key, value in shard.items():
            mapping[key] = name
            total += value.numel() * value.element_size()
    index = {"metadata": {"total_size": total}, "weight_map": mapping}
    tmp = path / "model.safetensors.index.json.tmp"
    tmp.write_text(json.dumps(index, indent=2))
    os.replace(tmp, path / "model.safetensors.index.json")
