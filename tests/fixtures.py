"""Tiny hybrid teachers and token datasets for CPU tests (no network, no HF forward)."""
import json
from pathlib import Path

import numpy as np
import torch

from rwkv_theseus_b200.config import DEFAULTS
from rwkv_theseus_b200.data import sha256_of_file
from rwkv_theseus_b200.models.hf_io import save_model
from rwkv_theseus_b200.models.qwen35 import HybridConfig, HybridForCausalLM


def tiny_config(depth=4, vocab=64):
    return HybridConfig(vocab_size=vocab, hidden_size=32, intermediate_size=64, num_hidden_layers=depth,
                        num_attention_heads=2, num_key_value_heads=1, head_dim=16,
                        linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=8,
                        linear_value_head_dim=8, linear_conv_kernel_dim=4,
                        layer_types=["linear_attention", "full_attention"] * (depth // 2),
                        rope_theta=10000.0, partial_rotary_factor=0.5)


def tiny_model(depth=4, seed=0, dtype=torch.bfloat16):
    torch.manual_seed(seed)
    model = HybridForCausalLM(tiny_config(depth)).init_weights()
    with torch.no_grad():  # non-trivial norms so the norm paths are exercised
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or name.endswith("_norm.weight"):
                p.normal_(0, 0.1)
    return model.to(dtype).eval().requires_grad_(False)


def save_tiny(path, depth=4, seed=0):
    model = tiny_model(depth, seed)
    save_model(model, path)
    return path


def write_dataset(path, vocab=64):
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    values = np.arange(37, dtype=np.uint32) % vocab
    values.tofile(path / "tokens.bin")
    np.save(path / "offsets.npy", np.array([0, 11, 28, 37], dtype=np.int64))
    manifest = {"format": 1, "vocab_size": vocab, "sources": [{
        "tokens": "tokens.bin", "offsets": "offsets.npy", "weight": 1,
        "tokens_sha256": sha256_of_file(path / "tokens.bin"), "offsets_sha256": sha256_of_file(path / "offsets.npy")}]}
    (path / "manifest.json").write_text(json.dumps(manifest))
    return path / "manifest.json"


# Run shape of the end-to-end CPU runs: 3-token chunks in 9-token windows, 3 steps per stage with 2 warm-up
# steps, two micro-steps per update, 2 validation chunks; logging every step, no periodic validation or checkpoints.
_RUN_SHAPE = {"chunk_tokens": 3, "context_tokens": 9, "stage_steps": 3, "warmup_steps": 2, "grad_accum_steps": 2,
              "validation_chunks": 2}
_CADENCE = {"log_interval": 1, "validation_interval": 0, "checkpoint_interval": 0}
_STUDENT = {"head_size": 8, "backend": "reference", "distributed_backend": "gloo", "training_mode": "sampled",
            "original_teacher_kl": True, "debug_input": True}


def make_config(tmp_path, stages):
    """A training config over a saved tiny teacher with `stages` attention blocks and two tiny token datasets."""
    save_tiny(tmp_path / "base", depth=stages * 2)
    paths = {"model": str(tmp_path / "base"), "output": str(tmp_path / "full"),
             "train_manifest": str(write_dataset(tmp_path / "train")),
             "validation_manifest": str(write_dataset(tmp_path / "val"))}
    cfg = {**DEFAULTS, **paths, **_STUDENT, **_RUN_SHAPE, **_CADENCE, "expected_attention_layers": stages}
    path = tmp_path / "config.json"
    path.write_text(json.dumps(cfg))
    return cfg, path
