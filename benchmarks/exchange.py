#!/usr/bin/env python3
"""Per-layer gradient exchange at the 27B TimeMix size (112.46 M fp32 parameters), one node.

Launch with torchrun, one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        benchmarks/exchange.py [--numel 112459520] [--iters 10]

Times (CUDA events, median of --iters after 3 warm-ups, max over ranks):
  peer  reduce-scatter + norm + clip + sharded AdamW + all-gather of the bf16 weight copy and the fp32
        non-decay parameters (``parallel.grad_sync``; NVLink bytes per rank and direction: (N-1)/N * 6n,
        4 bytes of fp32 gradient pulled, 2 bytes of bf16 weight pulled, small fp32 remainder ignored)
  nccl  NCCL all-reduce of the fp32 gradient + the full local clip/AdamW (the reference's scheme)
and reports the peer path against its NVLink roofline: those bytes at the measured 770 GB/s per
direction (the AdamW arithmetic is far below its compute bound).
"""
import argparse
import json
import os
import sys
import time
import types

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rwkv_theseus_b200.ops import native  # noqa: E402
from rwkv_theseus_b200.parallel.grad_sync import PeerGradExchange  # noqa: E402
from rwkv_theseus_b200.parallel.topology import Topology  # noqa: E402

LINK_GBS = 770.0


def student(n, dev):
    flat = types.SimpleNamespace(numel=n, param=torch.randn(n, device=dev) * 0.02, grad=torch.zeros(n, device=dev),
                                 exp_avg=torch.zeros(n, device=dev), exp_avg_sq=torch.zeros(n, device=dev))
    return types.SimpleNamespace(
        flat=flat, fused=types.SimpleNamespace(shadow=torch.zeros(n, device=dev, dtype=torch.bfloat16)),
        stats=torch.zeros(3, device=dev), report=torch.zeros(5, device=dev), decay_numel=n - 100_000,
        cfg={"betas": [0.9, 0.999], "adam_eps": 1e-8, "weight_decay": 0.01, "clip_norm": 1.0})


def timed(fn, iters, topo):
    out = []
    for i in range(iters + 3):
        topo.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        if i >= 3:
            out.append(s.elapsed_time(e))
    ms = torch.tensor([sorted(out)[len(out) // 2]], device=topo.device, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=topo.student_group)
    return ms.item()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--numel", type=int, default=112_459_520)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--blocks", default="148", help="comma-separated block counts to compare")
    p.add_argument("--profile", action="store_true")
    p.add_argument("--modes", default="split", help="comma-separated: split (update, then all-gather), fused")
    a = p.parse_args()
    topo = Topology("nccl", 5)
    dev, n, N = topo.device, a.numel, topo.world
    st = student(n, dev)
    ex = PeerGradExchange(topo, blocks=int(a.blocks.split(",")[0]), limit_s=60.0)
    ex.register(st)
    g = torch.randn(n, device=dev)
    step = [0]

    def peer():
        st.flat.grad.copy_(g)  # untimed part is excluded below by timing the copy alone
        st.stats.fill_(1.0)
        step[0] += 1
        ex.update(st, 1e-4, step[0])
        ex.wait()

    def copy_only():
        st.flat.grad.copy_(g)
        st.stats.fill_(1.0)

    norm2 = torch.zeros(native().flat_adamw_scratch(), device=dev)  # optimizer scratch (partial norms)

    def nccl():
        st.flat.grad.copy_(g)
        st.stats.fill_(1.0)
        dist.all_reduce(st.flat.grad, group=topo.student_group)
        dist.all_reduce(st.stats, group=topo.student_group)
        step[0] += 1
        native().flat_adamw(st.flat.param, st.flat.grad, st.flat.exp_avg, st.flat.exp_avg_sq, st.fused.shadow,
                            st.decay_numel, st.stats, norm2, st.report, 1e-4, 0.9, 0.999, 1e-8, 0.01, 1.0, step[0])

    if a.profile:  # per-kernel device times of the peer path (profiled run; not a benchmark number)
        from torch.profiler import ProfilerActivity, profile
        for _ in range(3):
            peer()
        topo.barrier()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(5):
                peer()
            torch.cuda.synchronize()
        topo.barrier()
        if topo.rank == 0:
            rows = {}
            for evt in prof.events():
                if evt.device_type == torch.autograd.DeviceType.CUDA:
                    rows.setdefault(evt.name[:48], []).append(evt.device_time)
            for name, ts in sorted(rows.items(), key=lambda kv: -sum(kv[1])):
                print(json.dumps({"kernel": name, "calls": len(ts), "avg_us": sum(ts) / len(ts)}), flush=True)
    from bench import ClockSampler  # nvidia-smi clocks and throttle reasons of this rank's GPU under load
    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    base = timed(copy_only, a.iters, topo)
    frac = (N - 1) / N
    link_ms = 6 * n * frac / (LINK_GBS * 1e9) * 1e3
    t_nccl = None
    results = []
    for mode in a.modes.split(","):
        ex.fused = mode == "fused"
        for blocks in [int(b) for b in a.blocks.split(",")]:
            ex.blocks = blocks
            t_peer = timed(peer, a.iters, topo) - base
            ex.check()
            if t_nccl is None:
                t_nccl = timed(nccl, a.iters, topo) - base
            results.append({"bench": "layer_exchange", "n_gpus": N, "numel": n, "peer_ms": t_peer,
                            "nccl_ms": t_nccl, "nvlink_roofline_ms": link_ms,
                            "peer_fraction_of_roofline": link_ms / t_peer, "speedup_vs_nccl": t_nccl / t_peer,
                            "blocks": blocks, "mode": mode})
    # The timed loops above last well under a second; the clock record comes from a separate 3-second loop of the
    # last configuration under nvidia-smi (its start-up stalls CUDA calls briefly, so it is not timed).
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    start = time.perf_counter()
    while True:
        peer()
        torch.cuda.synchronize()
        done = torch.tensor([time.perf_counter() - start > 3.0], device=dev, dtype=torch.int32)
        dist.all_reduce(done, op=dist.ReduceOp.MIN, group=topo.student_group)  # every rank leaves together
        if done.item():
            break
    clocks = sampler.stop()
    if topo.rank == 0:
        for line in results:
            print(json.dumps(line | {"clocks_rank0": clocks}), flush=True)
    ex.close()
    topo.close()


if __name__ == "__main__":
    main()
