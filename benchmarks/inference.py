#!/usr/bin/env python3
"""Assembled-model inference after migration (benchmark config e): the 27B hybrid with every
full-attention block replaced by its TimeMix student, bf16, random init. A batch of prompts of
uniform-random tokens is prefilled in chunks, then tokens are greedy-decoded with single-step
recurrent updates. Reports prefill tokens/s (CUDA events around the whole prefill) and the p50 / p90
per-token decode latency (CUDA events around every decode step), one GPU.

    python benchmarks/inference.py [--batch 8] [--prompt 4096] [--new 512] [--model 27b|small]
    python benchmarks/inference.py --impl reference [--new 64]

``--impl reference`` runs the unmodified reference package (installed under baseline/_ref): the random-init HF
Qwen3.5 model with the reference's TimeMix adapters installed by its own ``install`` and driven by its own
``Runner`` (reference ``theseus/inference.py:34-76`` returns that Runner from an export), greedy tokens from
``lm_head`` of the last hidden state. Same events, same prompt shape.
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from bench import MODEL_27B, MODEL_SMALL, layer_types  # noqa: E402
from rwkv_theseus_b200.inference import generate  # noqa: E402
from rwkv_theseus_b200.models.hf_io import random_model  # noqa: E402
from rwkv_theseus_b200.models.qwen35 import HybridConfig  # noqa: E402
from rwkv_theseus_b200.models.runner import Runner, install, migration_order  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--prompt", type=int, default=4096)
    p.add_argument("--new", type=int, default=512)
    p.add_argument("--prefill-chunk", type=int, default=4096)
    p.add_argument("--model", choices=("27b", "small"), default="27b")
    p.add_argument("--profile", action="store_true", help="per-kernel times of one decode step (profiled)")
    p.add_argument("--graph", action="store_true", help="replay the decode step as a CUDA graph")
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--profile-prefill", action="store_true",
                   help="after the timed run, per-kernel times of a second prefill (profiled)")
    a = p.parse_args()
    if a.impl == "reference":
        return run_reference(a)
    spec = MODEL_27B if a.model == "27b" else MODEL_SMALL
    cfg = HybridConfig(**spec, layer_types=layer_types(spec["num_hidden_layers"]))
    device = torch.device("cuda", 0)
    model = random_model(cfg, device, seed=0)
    order = migration_order(model, len([t for t in cfg.layer_types if t == "full_attention"]))
    for i, layer in enumerate(order):
        torch.manual_seed(i)
        install(model, layer, {"head_size": 64, "backend": "cuda", "lora_rank": None, "gate_lora_rank": None})
    runner = Runner(model)
    g = torch.Generator(device=device).manual_seed(7)
    prompt = torch.randint(0, cfg.vocab_size, (a.batch, a.prompt), device=device, generator=g)
    # warm-up: every kernel path once at the timed shapes (a full prefill chunk, then decode steps), so that the
    # GEMM tile choices are measured before the clock starts, as a serving process does once at start-up
    warm = torch.randint(0, cfg.vocab_size, (a.batch, min(a.prompt, a.prefill_chunk)), device=device, generator=g)
    generate(runner, warm, 4, prefill_chunk=a.prefill_chunk, graph=a.graph)
    torch.cuda.synchronize()
    events = []

    def on_token(step, ids):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        events.append(e)

    start, prefilled = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    original = runner.forward
    calls = {"n": 0}

    def forward(ids, *args, **kwargs):  # mark the end of prefill (first decode-sized call)
        if ids.shape[1] == 1 and calls["n"] == 0:
            prefilled.record()
            calls["n"] = 1
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append(e)
        return original(ids, *args, **kwargs)
    runner.forward = forward
    out = generate(runner, prompt, a.new, prefill_chunk=a.prefill_chunk, on_token=on_token, graph=a.graph)
    torch.cuda.synchronize()
    runner.forward = original
    prefill_ms = start.elapsed_time(prefilled)
    steps = sorted(events[i].elapsed_time(events[i + 1]) for i in range(2, len(events) - 1))  # skip the graph build
    result = {"bench": "assembled_inference", "model": f"qwen3.5-hybrid-{a.model} + {len(order)} TimeMix",
              "batch": a.batch, "prompt": a.prompt, "new_tokens": a.new, "dtype": "bf16",
              "prefill_tokens_per_s": a.batch * a.prompt / (prefill_ms / 1000), "prefill_ms": prefill_ms,
              "decode_p50_ms": steps[len(steps) // 2], "decode_p90_ms": steps[int(len(steps) * 0.9)],
              "decode_tokens_per_s": a.batch * 1000 / steps[len(steps) // 2], "generated": list(out.shape),
              "cuda_graph": a.graph,
              "data": "uniform-random prompt ids; random-init weights"}
    print(json.dumps(result), flush=True)
    if a.profile_prefill:
        from torch.profiler import ProfilerActivity, profile
        runner.reset()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for c in range(0, a.prompt, a.prefill_chunk):
                runner.forward(prompt[:, c:c + a.prefill_chunk])
            torch.cuda.synchronize()
        rows = {}
        for evt in prof.events():
            if evt.device_type == torch.autograd.DeviceType.CUDA:
                key = evt.name[:60]
                n, t = rows.get(key, (0, 0.0))
                rows[key] = (n + 1, t + evt.device_time)
        for name, (n, us) in sorted(rows.items(), key=lambda kv: -kv[1][1])[:25]:
            print(json.dumps({"prefill_kernel": name, "calls": n, "us": round(us, 1)}), flush=True)
    if a.profile:
        from torch.profiler import ProfilerActivity, profile
        token = out[:, -1:]
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            runner.forward(token)
            torch.cuda.synchronize()
        rows = {}
        for evt in prof.events():
            if evt.device_type == torch.autograd.DeviceType.CUDA:
                key = evt.name[:60]
                n, t = rows.get(key, (0, 0.0))
                rows[key] = (n + 1, t + evt.device_time)
        for name, (n, us) in sorted(rows.items(), key=lambda kv: -kv[1][1])[:25]:
            print(json.dumps({"kernel": name, "calls": n, "us": round(us, 1)}), flush=True)


def run_reference(a):
    if not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "theseus")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    from bench import reference_teacher
    from theseus.hf_model import Runner as RefRunner, install as ref_install, migration_order as ref_order
    spec = MODEL_27B if a.model == "27b" else MODEL_SMALL
    device = torch.device("cuda", 0)
    model = reference_teacher(spec, device)
    order = ref_order(model, len([t for t in model.config.layer_types if t == "full_attention"]))
    for i, layer in enumerate(order):
        torch.manual_seed(i)
        ref_install(model, layer, {"head_size": 64, "backend": "cuda"})
    runner = RefRunner(model)
    g = torch.Generator(device=device).manual_seed(7)
    prompt = torch.randint(0, model.config.vocab_size, (a.batch, a.prompt), device=device, generator=g)

    def greedy(hidden):
        return model.lm_head(hidden[:, -1]).argmax(-1, keepdim=True)

    warm = torch.randint(0, model.config.vocab_size, (a.batch, min(a.prompt, a.prefill_chunk)), device=device,
                         generator=g)
    tok = greedy(runner.forward(warm))
    for _ in range(3):
        tok = greedy(runner.forward(tok))
    runner.reset()
    torch.cuda.synchronize()
    start, prefilled = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    hidden = None
    for c in range(0, a.prompt, a.prefill_chunk):
        hidden = runner.forward(prompt[:, c:c + a.prefill_chunk])
    tok = greedy(hidden)
    prefilled.record()
    events = []
    for _ in range(a.new):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        events.append(e)
        tok = greedy(runner.forward(tok))
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    events.append(e)
    torch.cuda.synchronize()
    prefill_ms = start.elapsed_time(prefilled)
    steps = sorted(events[i].elapsed_time(events[i + 1]) for i in range(len(events) - 1))
    print(json.dumps({"bench": "assembled_inference", "impl": "reference",
                      "model": f"qwen3.5-hybrid-{a.model} + {len(order)} TimeMix (reference package)",
                      "batch": a.batch, "prompt": a.prompt, "new_tokens": a.new, "dtype": "bf16",
                      "prefill_tokens_per_s": a.batch * a.prompt / (prefill_ms / 1000), "prefill_ms": prefill_ms,
                      "decode_p50_ms": steps[len(steps) // 2], "decode_p90_ms": steps[int(len(steps) * 0.9)],
                      "decode_tokens_per_s": a.batch * 1000 / steps[len(steps) // 2],
                      "data": "uniform-random prompt ids; random-init weights"}), flush=True)


if __name__ == "__main__":
    main()
