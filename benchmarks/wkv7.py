#!/usr/bin/env python3
"""Standalone WKV7 recurrence benchmark.

bf16 inputs, fp32 state, B=8 lanes, T=4096 as 16 carried chunks of 256
tokens, H=40, N=64. r, k, v ~ N(0,1); decay exp(-exp(x)), x ~ U(-6, -0.5)
(expressed through the kernel's w input, decay = exp(-e^{-1/2} sigmoid(w)));
kk = L2-normalised N(0,1) per head, a = -kk, b = kk * sigmoid(N(0,1)).
Each chunk runs forward (state carried, detached) and backward. FLOPs use the
recurrence-equivalent count of the reference kernel: 9 N^2 forward + 24 N^2
backward per (batch, token, head). Device time with CUDA events; inputs
(>1 GB) exceed L2.

--impl ours       this package's chunked kernels
--impl reference  the reference project's kernels/wkv7_state.cu (JIT-built from baseline/_ref)
"""
import argparse
import json
import math
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def make_inputs(B, T, H, N, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    shape = (B, T, H, N)
    r = torch.randn(shape, device="cuda", generator=g)
    k = torch.randn(shape, device="cuda", generator=g)
    v = torch.randn(shape, device="cuda", generator=g)
    x = torch.rand(shape, device="cuda", generator=g) * 5.5 - 6.0          # U(-6, -0.5)
    p = torch.exp(x + 0.5).clamp(max=1 - 1e-6)                             # sigmoid(w) = e^x / e^{-1/2}
    w = torch.log(p) - torch.log1p(-p)
    kk = torch.nn.functional.normalize(torch.randn(shape, device="cuda", generator=g), dim=-1)
    a = -kk
    b = kk * torch.sigmoid(torch.randn(shape, device="cuda", generator=g))
    return [t.to(torch.bfloat16).contiguous() for t in (r, w, k, v, a, b)]


def ours_step_fn():
    sys.path.insert(0, ROOT)
    from rwkv_theseus_b200.ops import native
    ext = native()

    def run(xs, state, dy):
        y, end, ckpt, rec = ext.wkv7_forward(*xs, state, True)
        grads = ext.wkv7_backward(*xs, ckpt, rec, dy, torch.zeros_like(end))
        return end, grads
    return run


def reference_step_fn():
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    from theseus import wkv7 as ref  # unmodified reference module
    ext = ref.extension()

    def run(xs, state, dy):
        y, end, hist = ext.forward(*xs, state, True)
        grads = ext.backward(*xs, hist, dy, torch.zeros_like(end))
        return end, grads
    return run


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--B", type=int, default=8)
    p.add_argument("--T", type=int, default=4096)
    p.add_argument("--H", type=int, default=40)
    p.add_argument("--N", type=int, default=64)
    p.add_argument("--chunk", type=int, default=256)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=5)
    args = p.parse_args()
    B, T, H, N = args.B, args.T, args.H, args.N
    xs = make_inputs(B, T, H, N)
    dy = torch.randn_like(xs[0])
    step = ours_step_fn() if args.impl == "ours" else reference_step_fn()
    chunks = [(s, min(s + args.chunk, T)) for s in range(0, T, args.chunk)]
    sliced = [[x[:, a:b].contiguous() for x in xs] for a, b in chunks]
    dys = [dy[:, a:b].contiguous() for a, b in chunks]

    def one_pass():
        state = torch.zeros(B, H, N, N, device="cuda")
        for part, d in zip(sliced, dys):
            state, _ = step(part, state, d)
        return state

    for _ in range(args.warmup):
        one_pass()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.iters):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        one_pass()
        stop.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(stop))
    ms = sorted(times)[len(times) // 2]
    flops = 33.0 * N * N * B * T * H
    print(json.dumps({"metric": "wkv7 fwd+bwd", "impl": args.impl, "B": B, "T": T, "H": H, "N": N,
                      "chunk": args.chunk, "ms": ms, "tflops": flops / ms / 1e9, "dtype": "bf16",
                      "times_ms": times}))


if __name__ == "__main__":
    main()
