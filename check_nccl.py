#!/usr/bin/env python3
"""All-rank student preflight without loading the teacher (reference ``scripts/check_nccl.py``).

Runs two independent "stages" of --steps optimizer steps of a width-64 TimeMix student through the
framework's own update path (CUDA: fused kernels and, with more than one rank on a node, the
peer-memory gradient exchange; CPU/Gloo: the autograd path with all-reduce), with rank-dependent
sequence lengths (token-weighted reduction) and two micro-steps per update. After every step all
ranks must hold bit-identical parameters; each stage ends with the leader's weights broadcast to
every rank. Prints one JSON line per passed stage.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 check_nccl.py   # GPUs
    python -m torch.distributed.run --nproc-per-node 4 --master-addr 127.0.0.1 check_nccl.py --backend gloo
"""
import argparse
import hashlib
import json
import sys
import types
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from rwkv_theseus_b200.config import DEFAULTS  # noqa: E402
from rwkv_theseus_b200.parallel.topology import Topology  # noqa: E402
from rwkv_theseus_b200.stage import Student  # noqa: E402

WIDTH = 64


def fingerprint(student):
    h = hashlib.sha256()
    for name, value in sorted(student.weights().items()):
        h.update(name.encode())
        h.update(memoryview(value.detach().float().cpu().contiguous().view(torch.uint8).numpy()))
    return h.hexdigest()


def run(args):
    torch.set_num_threads(1)
    topo = Topology(args.backend, timeout_minutes=3)
    topo.assert_same(vars(args), "preflight arguments")
    cuda = topo.device.type == "cuda"
    cfg = DEFAULTS | {"head_size": 8, "backend": "cuda" if cuda else "reference", "lr": 1e-3,
                      "warmup_steps": 0, "grad_sync": args.grad_sync}
    model_cfg = types.SimpleNamespace(hidden_size=WIDTH, num_hidden_layers=2)
    for stage in range(2):
        torch.manual_seed(123 + stage)
        student = Student(model_cfg, stage, cfg, topo, total_steps=args.steps)
        topo.barrier()
        position = 0
        for step in range(args.steps):
            for micro in range(2):
                length = 3 + (topo.rank + step + micro) % 5  # rank-dependent lengths: token-weighted sums
                pos = torch.arange(position, position + length, device=topo.device, dtype=torch.float32)
                x = torch.sin(pos[None, :, None] + torch.arange(WIDTH, device=topo.device) / WIDTH)
                x = x.to(torch.bfloat16)
                target = (x.float() * 0.2 + 0.1).to(torch.bfloat16)
                student.micro_step(x, target)
                position += length
            student.reduce()
            student.update()
            topo.join_grad_sync()
            report = student.report.double().cpu().tolist()
            topo.check_grad_sync()
            if report[4] or report[2] <= 0:
                raise RuntimeError(f"invalid update on rank {topo.rank}: {report}")
            student.sync_state()
            prints = [None] * topo.world
            dist.all_gather_object(prints, fingerprint(student))
            if len(set(prints)) != 1:
                raise RuntimeError("Student parameters diverged after the update")
            for group in (student.flat.param, student.flat.exp_avg, student.flat.exp_avg_sq):
                assert group.dtype == torch.float32
        leader = topo.rank == topo.leader
        # the leader's bf16 weights reach every rank intact (the assembly path of validation and export)
        received = topo.broadcast_weights(
            {name: t.detach().cpu().to(torch.bfloat16) for name, t in student.weights().items()} if leader else None)
        if not received or any(t.dtype != torch.bfloat16 or not bool(t.isfinite().all()) for t in received.values()):
            raise RuntimeError("Broadcast weights arrived empty, in the wrong dtype or non-finite")
        if leader:
            sync = "local" if topo.world == 1 else (args.grad_sync if cuda else "all_reduce")
            record = {"stage": stage + 1, "backend": args.backend, "replicas": topo.world, "grad_sync": sync,
                      "steps": args.steps, "status": "passed"}
            print(json.dumps(record), flush=True)
        del student
        topo.barrier()
    topo.close()


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--backend", choices=("nccl", "gloo"), default="nccl")
    p.add_argument("--grad-sync", choices=("peer", "nccl"), default="peer",
                   help="multi-GPU gradient path on CUDA (peer-memory exchange or NCCL all-reduce)")
    p.add_argument("--steps", type=int, default=4)
    a = p.parse_args(argv)
    if a.steps < 1:
        p.error("steps must be positive")
    run(a)


if __name__ == "__main__":
    main()
