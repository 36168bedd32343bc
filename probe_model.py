#!/usr/bin/env python3
"""Single-GPU probe of a real teacher checkpoint (reference ``scripts/probe_model.py``); no training.

Loads the model, reports the migration order and memory, checks that one cached forward equals two
chunked forwards (final-hidden NMSE < 5e-3), and with --backward runs one student micro-step of the
first migrated layer on the captured pair and reports the statistics and peak memory.

    python probe_model.py --model ../Qwen3.8-27B [--tokens 16] [--backward]
"""
import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
import torch  # noqa: E402

from rwkv_theseus_b200.config import DEFAULTS  # noqa: E402
from rwkv_theseus_b200.losses import metrics, statistics  # noqa: E402
from rwkv_theseus_b200.models.hf_io import load_model  # noqa: E402
from rwkv_theseus_b200.models.runner import Capture, Runner, migration_order  # noqa: E402


class _LocalTopo:
    rank = world = 1
    leader = 0

    def __init__(self, device):
        self.rank, self.device = 0, device

    def grad_sync(self):
        return None


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", required=True)
    p.add_argument("--tokens", type=int, default=16)
    p.add_argument("--backward", action="store_true")
    a = p.parse_args(argv)
    torch.manual_seed(123)
    device = torch.device("cuda", 0)
    model = load_model(a.model, device)
    layers = [i for i, kind in enumerate(model.config.layer_types) if kind == "full_attention"]
    order = migration_order(model, len(layers))
    print(json.dumps({"loaded": True, "order": order, "allocated_gb": torch.cuda.memory_allocated() / 1e9}),
          flush=True)
    runner = Runner(model)
    capture = Capture(model.model.layers[order[0]].self_attn)
    ids = torch.randint(100, min(model.config.vocab_size, 1000), (1, a.tokens), device=device)
    full = runner.forward(ids).clone()
    x, y = capture.x.clone(), capture.y.clone()
    runner.reset()
    cut = a.tokens // 2
    chunked = torch.cat([runner.forward(ids[:, :cut]), runner.forward(ids[:, cut:])], 1)
    agreement = metrics(statistics(chunked.float(), full.float()))
    print(json.dumps({"chunk_equivalence": agreement}), flush=True)
    if agreement["nmse"] > 5e-3:
        raise RuntimeError("cached chunks deviate excessively from the one-shot forward")
    capture.close()
    if a.backward:
        from rwkv_theseus_b200.stage import Student
        cfg = DEFAULTS | {"head_size": 64, "backend": "cuda", "warmup_steps": 0}
        student = Student(model.config, order[0], cfg, _LocalTopo(device), total_steps=1)
        student.micro_step(x, y)
        grads = student.flat.grad
        if not torch.isfinite(grads).all() or not grads.abs().sum() > 0:
            raise RuntimeError("student backward produced no finite gradient")
        print(json.dumps({"backward": metrics(student.stats.detach().cpu()), "trainable_tensors":
                          len(student.flat.names), "peak_allocated_gb": torch.cuda.max_memory_allocated() / 1e9}),
              flush=True)


if __name__ == "__main__":
    main()
