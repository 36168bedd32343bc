#!/usr/bin/env python3
"""tcgen05 flash attention vs PyTorch SDPA on the 27B layer shape: 1024 queries of 24 heads (head_dim 256,
4 KV heads) at cache offsets 0/1024/2048/3072 (the four chunks of a 4096-token window). CUDA-event timing of
10 back-to-back launches per sample (so the host's launch preparation overlaps the previous launch instead of
being timed), median of 20 samples after 5 warm-ups; FLOPs count the causal work only."""
import json
import os
import sys

import torch
from torch.nn import functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rwkv_theseus_b200.ops import native  # noqa: E402


REPEAT = 10


def timed(fn, warmup=5, iters=20):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(REPEAT):
            fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e) / REPEAT)
    return sorted(out)[len(out) // 2]


def main():
    B, T, Hq, Hkv, D, cap = 1, 1024, 24, 4, 256, 4096
    for offset in (0, 1024, 2048, 3072):
        L = offset + T
        q = torch.randn(B, T, Hq, D, device="cuda").to(torch.bfloat16)
        keys = torch.randn(B, cap, Hkv, D, device="cuda").to(torch.bfloat16)
        values = torch.randn_like(keys)
        qg = torch.randn(B * T, Hq * 2 * D, device="cuda").to(torch.bfloat16)
        mask = torch.arange(L, device="cuda")[None] <= (torch.arange(T, device="cuda")[:, None] + offset)

        def ours():
            native().flash_attention(q, keys, values, qg, offset)

        def sdpa():
            o = F.scaled_dot_product_attention(q.transpose(1, 2), keys[:, :L].transpose(1, 2),
                                               values[:, :L].transpose(1, 2), attn_mask=mask, scale=D ** -0.5,
                                               enable_gqa=True)
            o.transpose(1, 2) * torch.sigmoid(qg.view(B, T, Hq, 2 * D)[..., D:])

        flops = 4.0 * B * Hq * D * T * (offset + (T + 1) / 2)
        t_ours, t_sdpa = timed(ours), timed(sdpa)
        print(json.dumps({"offset": offset, "ours_ms": t_ours, "sdpa_ms": t_sdpa,
                          "ours_tflops": flops / t_ours / 1e9, "sdpa_tflops": flops / t_sdpa / 1e9}), flush=True)


if __name__ == "__main__":
    main()
