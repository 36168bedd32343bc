#!/usr/bin/env python3
"""tcgen05 GEMM vs cuBLAS (torch.matmul) on the projection shapes of the 27B
migration step (1024 tokens): teacher MLP/GDN/attention projections and the
student C x C GEMMs in forward, input-gradient (MN-major B) and
weight-gradient (MN-major A and B) form. Rows with G = 3 are the student's
r/k/v projections as one grouped launch (``gemm_group``) against one batched
cuBLAS call (``torch.bmm``) on the same operands. Device time with CUDA events,
median of --iters after --warmup; operands rotate over buffers larger than L2.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rwkv_theseus_b200.ops import native  # noqa: E402

SHAPES = [  # (name, M, N, K, a_t, b_t[, G])
    ("mlp_gate_up", 1024, 17408, 5120, False, False),
    ("mlp_down", 1024, 5120, 17408, False, False),
    ("gdn_in_qkv", 1024, 10240, 5120, False, False),
    ("gdn_out", 1024, 5120, 6144, False, False),
    ("attn_q", 1024, 12288, 5120, False, False),
    ("student_fwd", 1024, 5120, 5120, False, False),
    ("student_dx", 1024, 5120, 5120, False, True),
    ("student_dw", 5120, 5120, 1024, True, True),
    ("student_rkv_fwd", 1024, 5120, 5120, False, False, 3),
    ("student_rkv_dx", 1024, 5120, 5120, False, True, 3),
    ("student_rkv_dw", 5120, 5120, 1024, True, True, 3),
    ("mlp_swiglu", 1024, 17408, 5120, False, False, "swiglu"),
    ("lora_down", 1024, 192, 5120, False, False),
    ("gdn_ab", 1024, 96, 5120, False, False),
    ("big_square", 8192, 8192, 8192, False, False),
]


def timed(fn, warmup, iters):
    for _ in range(warmup):
        fn(0)
    torch.cuda.synchronize()
    times = []
    for i in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn(i + 1)
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return sorted(times)[len(times) // 2]


def bench_swiglu(name, M, N, K, args, tile):
    """silu(x Wg^T) * (x Wu^T) in one launch against two cuBLAS GEMMs and the eager elementwise product."""
    import torch.nn.functional as F
    sets = 2
    xs = [torch.randn(M, K, device="cuda").to(torch.bfloat16) for _ in range(sets)]
    ws = [(torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16) for _ in range(2 * sets)]

    def ours(i):
        return native().gemm_swiglu(xs[i % sets], ws[2 * (i % sets)], ws[2 * (i % sets) + 1], tile)

    def cublas(i):
        x = xs[i % sets]
        return F.silu(x @ ws[2 * (i % sets)].t()) * (x @ ws[2 * (i % sets) + 1].t())

    flops = 4.0 * M * N * K
    t_ours = timed(ours, args.warmup, args.iters)
    t_cub = float("nan") if args.no_cublas else timed(cublas, args.warmup, args.iters)
    ref = (F.silu(xs[0].float() @ ws[0].float().t()) * (xs[0].float() @ ws[1].float().t()))
    rel = ((ours(0).float() - ref).abs().max() / ref.abs().max()).item()
    row = {"shape": name, "M": M, "N": N, "K": K, "G": 2, "ours_ms": t_ours, "cublas_ms": t_cub,
           "ours_tflops": flops / t_ours / 1e9, "cublas_tflops": flops / t_cub / 1e9, "ratio": t_cub / t_ours,
           "max_rel_err": rel}
    print(json.dumps(row), flush=True)
    return row


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--only", default=None)
    p.add_argument("--tile", default=None,
                   help="fixed tile choice instead of the measured one: width, then 'm2' for 256-row tiles, 'sk' for "
                        "stream-K or 'spS' for parallel split-K over S CTAs per tile (e.g. 256sk, 256m2sk, 64sp16)")
    p.add_argument("--no-cublas", action="store_true")
    args = p.parse_args()
    tile = 0
    if args.tile:
        spec = args.tile
        if "sp" in spec:
            spec, parts = spec.split("sp")
            tile |= int(parts) << 20
        if spec.endswith("sk"):
            spec, tile = spec[:-2], tile | (1 << 16)
        if spec.endswith("m2"):
            spec, tile = spec[:-2], tile | (1 << 17)
        tile |= int(spec)
    results = []
    for name, M, N, K, a_t, b_t, *rest in SHAPES:
        if args.only and args.only not in name:
            continue
        swiglu = bool(rest) and rest[0] == "swiglu"
        G = rest[0] if rest and not swiglu else 1
        if swiglu:
            results.append(bench_swiglu(name, M, N, K, args, tile))
            continue
        bytes_per_set = G * (M * K + N * K) * 2
        sets = max(1, min(8, (256 << 20) // bytes_per_set + 1))
        As = [torch.randn((G, K, M) if a_t else (G, M, K), device="cuda").to(torch.bfloat16) for _ in range(sets)]
        Bs = [torch.randn((G, K, N) if b_t else (G, N, K), device="cuda").to(torch.bfloat16) for _ in range(sets)]
        out = torch.empty(G, M, N, device="cuda", dtype=torch.bfloat16)
        outs = list(out.unbind(0))

        def ours(i):
            if G == 1:
                native().gemm(As[i % sets][0], a_t, Bs[i % sets][0], b_t, 0, 1.0, out[0], tile)
            else:
                native().gemm_group(list(As[i % sets].unbind(0)), a_t, list(Bs[i % sets].unbind(0)), b_t, 0, 1.0,
                                    outs, tile)

        def cublas(i):
            a = As[i % sets].transpose(1, 2) if a_t else As[i % sets]
            b = Bs[i % sets] if b_t else Bs[i % sets].transpose(1, 2)
            if G == 1:
                torch.matmul(a[0], b[0], out=out[0])
            else:
                torch.bmm(a, b, out=out)

        flops = 2.0 * M * N * K * G
        t_ours = timed(ours, args.warmup, args.iters)
        t_cub = float("nan") if args.no_cublas else timed(cublas, args.warmup, args.iters)
        ref = torch.matmul(As[0].transpose(1, 2) if a_t else As[0], Bs[0] if b_t else Bs[0].transpose(1, 2)).float()
        ours(0)
        rel = ((out.float() - ref).abs().max() / ref.abs().max()).item()
        row = {"shape": name, "M": M, "N": N, "K": K, "G": G, "ours_ms": t_ours, "cublas_ms": t_cub,
               "ours_tflops": flops / t_ours / 1e9, "cublas_tflops": flops / t_cub / 1e9,
               "ratio": t_cub / t_ours, "max_rel_err": rel}
        results.append(row)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
