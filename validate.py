#!/usr/bin/env python3
"""Standalone validation of a committed checkpoint with all-rank metric reduction.

Complete parallel checkpoints get composition validation, incomplete ones
parallel (teacher-forced) validation, legacy sequential ones the single-stage
validation.
"""
import argparse
import json

from rwkv_theseus_b200.checkpoint import model_fingerprint, read_checkpoint
from rwkv_theseus_b200.config import load_config
from rwkv_theseus_b200.models.hf_io import load_model
from rwkv_theseus_b200.models.runner import Capture, Runner, install
from rwkv_theseus_b200.parallel.topology import Topology
from rwkv_theseus_b200.stage import Student
from rwkv_theseus_b200.validation import validate, validate_composition, validate_parallel

if __name__ == "__main__":
    p = argparse.ArgumentParser()
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", required=True)
    args = p.parse_args()
    cfg = load_config(args.config)
    topo = Topology(cfg["distributed_backend"], cfg["timeout_minutes"])
    topo.assert_same({"config": cfg, "checkpoint": args.checkpoint}, "validation configuration")
    _, meta, delta = read_checkpoint(args.checkpoint)
    if meta["base_fingerprint"] != model_fingerprint(cfg["model"]):
        raise ValueError("Validation base differs from training")
    model = load_model(cfg["model"], topo.device)
    if meta.get("training_topology") == "parallel_layers_v1":
        if meta["complete"]:
            for layer in meta["order"]:
                install(model, layer, cfg, delta[layer])
            results = validate_composition(topo, cfg, Runner(model))
        else:
            students = {layer: Student(model.config, layer, cfg, topo, delta[layer]) for layer in meta["order"]}
            captures = {layer: Capture(model.model.layers[layer].self_attn) for layer in meta["order"]}
            try:
                results = validate_parallel(topo, cfg, Runner(model), students, captures)
            finally:
                for capture in captures.values():
                    capture.close()
    else:
        for layer in meta["order"][:meta["stage"]]:
            install(model, layer, cfg, delta[layer])
        layer = meta["order"][meta["stage"]]
        install(model, layer, cfg, delta[layer], trainable=True, retain_teacher=True)
        model.requires_grad_(False)
        results = validate(topo, cfg, Runner(model), layer)
    if topo.rank == topo.leader:
        print(json.dumps(results, indent=2))
    topo.close()
