#!/usr/bin/env python3
"""Per-layer recurrent kernels at the 27B migration shapes (one 1024-token chunk):
GDN forward (48 value / 16 key heads, head size 128) and WKV7 forward + backward (80 heads of 64).
CUDA-event timing, median of --iters after --warmup."""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rwkv_theseus_b200.ops import native  # noqa: E402


def timed(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return sorted(out)[len(out) // 2]


def kernel_times(fn, reps=3):
    """Per-kernel device time (us per call) from a profiled run; not a benchmark number."""
    from torch.profiler import ProfilerActivity, profile
    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    rows = {}
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA:
            rows[evt.name[:60]] = rows.get(evt.name[:60], 0.0) + evt.device_time / reps
    for name, us in sorted(rows.items(), key=lambda kv: -kv[1]):
        print(json.dumps({"kernel": name, "us_per_call": round(us, 1)}), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--T", type=int, default=1024)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--only", default=None)
    p.add_argument("--profile", action="store_true", help="also print per-kernel device times (profiled run)")
    a = p.parse_args()
    ext = native()
    T = a.T
    if a.only in (None, "gdn"):
        Hk, Hv, D = 16, 48, 128
        qkv = (torch.randn(1, T, 2 * Hk * D + Hv * D, device="cuda") * 0.5).to(torch.bfloat16)
        ab = torch.randn(T, 2 * Hv, device="cuda").to(torch.bfloat16)
        A_log, dt = torch.rand(Hv, device="cuda") * 3, torch.randn(Hv, device="cuda")
        state = torch.zeros(1, Hv, D, D, device="cuda")
        fn = lambda: ext.gdn_forward(qkv, ab[:, :Hv], ab[:, Hv:], A_log, dt, state, Hk, Hv, D)  # noqa: E731
        ms = timed(fn, a.warmup, a.iters)
        print(json.dumps({"kernel": "gdn_forward", "T": T, "ms": ms}), flush=True)
        if a.profile:
            kernel_times(fn)
    if a.only in (None, "wkv"):
        B, H, N = 1, 80, 64
        xs = [torch.randn(B, T, H, N, device="cuda").to(torch.bfloat16) for _ in range(6)]
        s0 = torch.zeros(B, H, N, N, device="cuda")
        fwd = lambda: ext.wkv7_forward(*xs, s0, True)  # noqa: E731
        ms = timed(fwd, a.warmup, a.iters)
        print(json.dumps({"kernel": "wkv7_forward", "T": T, "ms": ms}), flush=True)
        if a.profile:
            kernel_times(fwd)
        y, end, ck, rec = ext.wkv7_forward(*xs, s0, True)
        dy, dend = torch.randn_like(y), torch.zeros_like(end)
        bwd = lambda: ext.wkv7_backward(*xs, ck, rec, dy, dend)  # noqa: E731
        ms = timed(bwd, a.warmup, a.iters)
        print(json.dumps({"kernel": "wkv7_backward", "T": T, "ms": ms}), flush=True)
        if a.profile:
            kernel_times(bwd)


if __name__ == "__main__":
    main()
