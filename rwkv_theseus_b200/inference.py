"""Self-contained export of the assembled model and its runtime.

Export format 2 (reference ``theseus/inference.py:14-31``): HF-layout sharded
safetensors (5 GB shards) in which every migrated block's TimeMix weights sit
under ``model.layers.<i>.self_attn.core.*`` in bf16, ``config.json``, the
tokenizer files of the base model, and ``theseus.json`` =
``{format: 2, layers, head_size, backend, base_fingerprint, loader,
state_layout: "B,H,value,key", migration_fingerprint}``.

``load_export`` rebuilds the model on the meta device, installs the TimeMix
blocks, loads the shards strictly and returns a ``Runner``. Format-1 exports
(base model + delta) are also accepted. ``generate`` adds the greedy decode
loop the reference leaves to the caller: one chunked prefill, then T=1 steps
through the recurrent states (WKV7/GDN) and the KV cache.
"""
import json
import os
import shutil
from pathlib import Path

import torch
from safetensors.torch import load_file

from .checkpoint import model_fingerprint, split_delta
from .data import sha256_of_file
from .models.hf_io import build_empty, finalize, load_model, save_model, shard_files
from .models.qwen35 import HybridConfig
from .models.runner import Runner, install

TOKENIZER_PREFIXES = ("tokenizer", "vocab", "merges", "special_tokens", "chat_template")


def save_export(model, path, cfg, order, base_id, checkpoint=None):
    path = Path(path)
    if path.exists():
        raise FileExistsError(f"Refusing to overwrite export {path}")
    temp = path.with_name("." + path.name + ".tmp")
    if temp.exists():
        shutil.rmtree(temp)
    temp.mkdir(parents=True)
    save_model(model, temp, max_shard_bytes=5 * 1000 ** 3)
    for source in Path(cfg["model"]).iterdir():
        if source.is_file() and source.name.startswith(TOKENIZER_PREFIXES):
            shutil.copyfile(source, temp / source.name)
    meta = {"format": 2, "layers": order, "head_size": cfg["head_size"], "backend": cfg["backend"],
            "lora_rank": cfg.get("lora_rank"), "gate_lora_rank": cfg.get("gate_lora_rank"),
            "base_fingerprint": base_id, "loader": "rwkv_theseus_b200.inference.load_export",
            "state_layout": "B,H,value,key",
            "migration_fingerprint": sha256_of_file(Path(checkpoint) / "migrated.safetensors") if checkpoint else None}
    (temp / "theseus.json").write_text(json.dumps(meta, indent=2))
    os.replace(temp, path)


def _load_full_export(root, meta, device):
    """Format 2: a complete converted model directory (config + bf16 shards, migrated layers named
    ``model.layers.<i>.self_attn.core.*``). Every expected tensor must come from exactly one shard."""
    cfg = HybridConfig.from_pretrained(root)
    model = build_empty(cfg, "meta", torch.bfloat16)
    for layer in meta["layers"]:
        install(model, layer, meta)
    wanted = set(model.state_dict())
    loaded = set()
    for shard in shard_files(root):
        tensors = load_file(str(root / shard), device=str(device))
        names = set(tensors)
        if names - wanted or names & loaded:
            raise ValueError(f"Invalid converted checkpoint keys in {shard}")
        model.load_state_dict(tensors, strict=False, assign=True)
        loaded |= names
    if cfg.tie_word_embeddings and "lm_head.weight" not in loaded:
        model.lm_head.weight = model.model.embed_tokens.weight
        loaded.add("lm_head.weight")
    missing = sorted(wanted - loaded)
    if missing:
        raise ValueError(f"Missing converted weights: {missing[:8]}")
    finalize(model, device)
    return model


def _load_delta_export(root, meta, device, base_model):
    """Format 1: the migrated TimeMix tensors only, installed into the original base model, whose fingerprint
    must match the one recorded at export."""
    base = base_model if base_model else meta["base_model"]
    if meta["base_fingerprint"] != model_fingerprint(base):
        raise ValueError("Export base fingerprint mismatch")
    model = load_model(base, device)
    per_layer = split_delta(load_file(str(root / "migrated.safetensors")))
    for layer in meta["layers"]:
        install(model, layer, meta, per_layer[layer])
    return model


def load_export(path, device="cuda", base_model=None):
    """A ``Runner`` over the assembled model of an export directory (format 2, or the delta-only format 1)."""
    root = Path(path)
    meta = json.loads((root / "theseus.json").read_text())
    if meta["format"] == 2:
        return Runner(_load_full_export(root, meta, device))
    return Runner(_load_delta_export(root, meta, device, base_model))


@torch.no_grad()
class DecodeGraph:
    """One greedy decode step (T = 1 forward, lm_head, argmax) captured as a CUDA graph.

    Built after an eager decode step, so every recurrent state exists in its final shape. The GDN conv
    windows / delta-rule states and the TimeMix shift / WKV states are kept in persistent buffers: the
    captured step reads them, and copies the new states back into them at its end (the delta-rule state is
    already updated in place). Replays therefore advance exactly like eager steps; the host only writes the
    input token and advances the cache cursor. Needs a model whose attention blocks are all replaced (no KV
    cache grows during decoding).
    """

    def __init__(self, runner, token):
        from .models.runner import AttentionAdapter
        model = runner.model
        layers = model.model.layers
        if any(kind == "full_attention" and not isinstance(getattr(layers[i], "self_attn", None), AttentionAdapter)
               for i, kind in enumerate(model.config.layer_types)):
            raise ValueError("graph decoding needs every full-attention block replaced by a TimeMix")
        self.runner = runner
        self.ids = token.clone()
        head = model.lm_head.weight
        self.gdn = [(layer, layer["conv"], layer["recurrent"]) for layer in runner.cache.layers if "recurrent" in layer]
        self.adapters = [(b.self_attn, {k: v.clone() for k, v in b.self_attn.state.items()})
                         for b in layers if isinstance(getattr(b, "self_attn", None), AttentionAdapter)]
        for adapter, persistent in self.adapters:
            adapter.state = persistent
        cursor = runner.cache.cursor
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side), torch.cuda.graph(self.graph):
            hidden = runner.forward(self.ids)
            self.out = (hidden[:, -1:].to(head.dtype) @ head.t()).argmax(-1)
            for layer, conv, rec in self.gdn:
                if layer["conv"] is not conv:
                    conv.copy_(layer["conv"])
                if layer["recurrent"] is not rec:
                    rec.copy_(layer["recurrent"])
            for adapter, persistent in self.adapters:
                for key, value in persistent.items():
                    value.copy_(adapter.state[key])
        torch.cuda.current_stream().wait_stream(side)
        # capture ran nothing: point the Python-side state at the persistent buffers again
        for layer, conv, rec in self.gdn:
            layer["conv"], layer["recurrent"] = conv, rec
        for adapter, persistent in self.adapters:
            adapter.state = persistent
        runner.cache.cursor = cursor

    def step(self, token):
        self.ids.copy_(token)
        self.graph.replay()
        self.runner.cache.cursor += 1
        return self.out.clone()


def generate(runner, prompt, new_tokens, prefill_chunk=4096, on_token=None, graph=False):
    """Greedy decoding: chunked prefill of ``prompt`` [B, T], then ``new_tokens`` T=1 steps.

    Returns the generated ids [B, new_tokens]. ``on_token(step, ids)`` is called
    after each decode step (timing hooks, streaming). ``graph=True`` replays the
    decode step as a CUDA graph after the first eager step (assembled models).
    """
    runner.reset()
    head = runner.model.lm_head.weight
    hidden = None
    for start in range(0, prompt.shape[1], prefill_chunk):
        hidden = runner.forward(prompt[:, start:start + prefill_chunk])
    token = (hidden[:, -1:].to(head.dtype) @ head.t()).argmax(-1)
    out = [token]
    stepper = None
    for step in range(1, new_tokens):
        if stepper is not None:
            token = stepper.step(token)
        else:
            hidden = runner.forward(token)
            token = (hidden[:, -1:].to(head.dtype) @ head.t()).argmax(-1)
            if graph and step + 1 < new_tokens:
                stepper = DecodeGraph(runner, token)
        out.append(token)
        if on_token is not None:
            on_token(step, token)
    return torch.cat(out, 1)
