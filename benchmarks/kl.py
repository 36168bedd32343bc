#!/usr/bin/env python3
"""Validation KL over the vocabulary: one-pass kernel (csrc/fused/kl.cu) vs two log_softmax passes in PyTorch
(the reference's kl_sum). Rows = kl_token_block tokens x batch, vocabulary of the 27B config; bf16 logits as
lm_head produces them. Device time with CUDA events, median of --iters after --warmup.

    python benchmarks/kl.py [--rows 16] [--vocab 248077]
"""
import argparse
import json
import os
import sys

import torch
from torch.nn import functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rwkv_theseus_b200.ops import native  # noqa: E402


def timed(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return sorted(times)[len(times) // 2]


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--rows", type=int, default=16)
    p.add_argument("--vocab", type=int, default=248077)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    a = p.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    s = (torch.randn(a.rows, a.vocab, device="cuda", generator=g) * 3).to(torch.bfloat16)
    t = (s.float() + torch.randn(a.rows, a.vocab, device="cuda", generator=g)).to(torch.bfloat16)

    def torch_kl():
        lt, ls = F.log_softmax(t.float(), -1), F.log_softmax(s.float(), -1)
        return (lt.exp() * (lt - ls)).sum()

    ours = timed(lambda: native().kl_rows(s, t), a.warmup, a.iters)
    ref = timed(torch_kl, a.warmup, a.iters)
    err = abs(native().kl_rows(s, t).sum().item() - torch_kl().item()) / abs(torch_kl().item())
    moved = 2 * s.numel() * s.element_size()
    print(json.dumps({"bench": "kl_rows", "rows": a.rows, "vocab": a.vocab, "ours_ms": ours, "torch_ms": ref,
                      "speedup": ref / ours, "hbm_gbs": moved / ours / 1e6, "rel_err": err}), flush=True)


if __name__ == "__main__":
    main()
