#!/usr/bin/env python3
"""Compose a completed migration checkpoint into a self-contained full model."""
import argparse

from rwkv_theseus_b200.checkpoint import model_fingerprint, read_checkpoint
from rwkv_theseus_b200.inference import save_export
from rwkv_theseus_b200.models.hf_io import load_model
from rwkv_theseus_b200.models.runner import install

if __name__ == "__main__":
    p = argparse.ArgumentParser()
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--output", required=True)
    args = p.parse_args()
    checkpoint, meta, delta = read_checkpoint(args.checkpoint)
    if not meta["complete"] or set(delta) != set(meta["order"]):
        raise ValueError("Final export requires all layers to have completed training")
    cfg = meta["config"]
    if model_fingerprint(cfg["model"]) != meta["base_fingerprint"]:
        raise ValueError("Base weights changed")
    model = load_model(cfg["model"], "cpu")
    for layer in meta["order"]:
        install(model, layer, cfg, delta[layer])
    save_export(model, args.output, cfg, meta["order"], meta["base_fingerprint"], checkpoint=checkpoint)
    print(args.output)
