#!/usr/bin/env python3
"""Host issue time against device time of one eager fused TimeMix micro-step at the 27B student shape
(C 5120, 80 heads of 64), for full and partial chunks. The eager path runs for the shorter last chunk of every
document (full chunks replay a CUDA graph), so when its host issue time exceeds its device time the GPU waits.

    python benchmarks/student_step.py [--tokens 1024,512,300] [--iters 5] [--profile]

host_ms: wall time for the micro-step call to return (launches queued, nothing waited for), device_ms: CUDA
events around it. --profile adds the host-side op table of one call (torch.profiler, CPU activity only).
"""
import argparse
import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rwkv_theseus_b200.config import DEFAULTS  # noqa: E402
from rwkv_theseus_b200.models.qwen35 import HybridConfig  # noqa: E402
from rwkv_theseus_b200.stage import Student  # noqa: E402


class _Topo:
    def __init__(self, device):
        self.rank, self.world, self.leader, self.device = 0, 1, 0, device

    def grad_sync(self):
        return None


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", default="1024,512,300")
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--profile", action="store_true")
    args = p.parse_args()
    device = torch.device("cuda", 0)
    cfg = HybridConfig(vocab_size=1024, hidden_size=5120, intermediate_size=1024, num_hidden_layers=64,
                       num_attention_heads=24, num_key_value_heads=4, head_dim=256, linear_num_key_heads=16,
                       linear_num_value_heads=48, linear_key_head_dim=128, linear_value_head_dim=128,
                       linear_conv_kernel_dim=4, layer_types=["linear_attention", "full_attention"] * 32)
    train = DEFAULTS | {"head_size": 64, "backend": "cuda", "student_graphs": False}
    student = Student(cfg, 3, train, _Topo(device), total_steps=10)
    for T in [int(t) for t in args.tokens.split(",")]:
        x = torch.randn(1, T, cfg.hidden_size, device=device).to(torch.bfloat16)
        y = torch.randn(1, T, cfg.hidden_size, device=device).to(torch.bfloat16)
        for _ in range(2):  # tile choices measured, allocator warm
            student.state = None
            student.micro_step(x, y)
        torch.cuda.synchronize()
        hosts, devs = [], []
        for _ in range(args.iters):
            student.state = None
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            start.record()
            t0 = time.perf_counter()
            student.micro_step(x, y)
            hosts.append((time.perf_counter() - t0) * 1e3)
            stop.record()
            torch.cuda.synchronize()
            devs.append(start.elapsed_time(stop))
        print(json.dumps({"tokens": T, "host_ms": sorted(hosts)[len(hosts) // 2],
                          "device_ms": sorted(devs)[len(devs) // 2]}), flush=True)
        if args.profile:
            from torch.profiler import ProfilerActivity, profile
            with profile(activities=[ProfilerActivity.CPU]) as prof:
                student.state = None
                student.micro_step(x, y)
            torch.cuda.synchronize()
            print(prof.key_averages().table(sort_by="self_cpu_time_total", row_limit=25), flush=True)


if __name__ == "__main__":
    main()
