"""Process topology: Gloo world group for control, NCCL group for data.

Same contract as the reference ``theseus/distributed.py:11-111``: torchrun
environment, one GPU per local rank, a Gloo world process group carrying
configuration agreement, barriers and object broadcasts, and one student group
(NCCL on GPUs, Gloo in CPU tests) warmed with an all-reduce before any large
allocation. Ranks that report inconsistent facts or share a GPU are rejected.

On top of that the topology owns the per-node peer-memory gradient exchange
(``parallel.grad_sync``), created lazily when the student group is NCCL and
all ranks sit on one NVSwitch node.
"""
from datetime import timedelta
import hashlib
import json
import os
import socket

import torch
import torch.distributed as dist


def _env_int(name, default=None):
    value = os.environ.get(name)
    if value is None:
        if default is None:
            raise KeyError(f"{name} is not set; launch with torchrun")
        return default
    return int(value)


class Topology:
    def __init__(self, backend="nccl", timeout_minutes=60):
        self.rank = _env_int("RANK")
        self.world = _env_int("WORLD_SIZE")
        self.local_rank = _env_int("LOCAL_RANK")
        local_world = _env_int("LOCAL_WORLD_SIZE", self.world)
        self.local_world = local_world
        if self.world < 1 or local_world < 1 or self.world % local_world or self.local_rank != self.rank % local_world:
            raise ValueError("Use uniform torchrun rank allocation")
        self.backend = backend
        if backend == "nccl":
            if not torch.cuda.is_available() or torch.cuda.device_count() < local_world:
                raise RuntimeError("Need one visible GPU per local rank")
            torch.cuda.set_device(self.local_rank)
            self.device = torch.device("cuda", self.local_rank)
            if not torch.cuda.is_bf16_supported():
                raise RuntimeError("BF16-capable GPUs are required")
        elif backend == "gloo":
            self.device = torch.device("cpu")
        else:
            raise ValueError(backend)
        self.timeout = timedelta(minutes=timeout_minutes)
        if not dist.is_initialized():
            dist.init_process_group("gloo", timeout=self.timeout)
        facts = (local_world, backend, socket.gethostname(),
                 str(torch.cuda.get_device_properties(self.device).uuid) if backend == "nccl" else None)
        reports = [None] * self.world
        dist.all_gather_object(reports, facts)
        if any(tuple(r[:2]) != facts[:2] for r in reports):
            raise ValueError("Inconsistent rank configuration")
        devices = [tuple(r[2:]) for r in reports if r[3] is not None]
        if len(devices) != len(set(devices)):
            raise ValueError("Multiple ranks share a GPU")
        self.single_node = len({r[2] for r in reports}) == 1
        self.students = list(range(self.world))
        self.leader = 0
        self.groups = []
        self.tracker = None
        self.student_group = self._create_group(self.students)
        self._grad_sync = None

    def _create_group(self, ranks):
        group = dist.new_group(ranks, backend=self.backend, timeout=self.timeout)
        self.groups.append(group)
        if self.rank in ranks:
            probe = torch.ones(1, device=self.device)
            dist.all_reduce(probe, group=group)
            self.synchronize()
            if probe.item() != len(ranks):
                raise RuntimeError("Process group warm-up failed")
        dist.barrier()
        return group

    def synchronize(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def barrier(self):
        self.synchronize()
        dist.barrier()

    def close(self):
        self.barrier()
        if self._grad_sync is not None:
            self._grad_sync.close()
            self._grad_sync = None
        dist.destroy_process_group()

    def assert_same(self, value, label):
        digest = hashlib.sha256(json.dumps(value, sort_keys=True, default=str).encode()).hexdigest()
        gathered = [None] * self.world
        dist.all_gather_object(gathered, digest)
        if len(set(gathered)) != 1:
            raise ValueError(f"Ranks disagree on {label}: {gathered}")

    def student_sum(self, tensor):
        """In-place sum over the student group on the current stream."""
        if self.world > 1:
            dist.all_reduce(tensor, group=self.student_group)
        return tensor

    def broadcast_object(self, value, source=None):
        self.synchronize()
        box = [value]
        dist.broadcast_object_list(box, src=self.leader if source is None else source)
        return box[0]

    def broadcast_weights(self, state):
        """Leader's tensors to every rank as raw bytes, then a digest agreement."""
        self.barrier()
        spec = None
        if self.rank == self.leader:
            spec = [(name, tuple(v.shape), str(v.dtype).removeprefix("torch.")) for name, v in sorted(state.items())]
        spec = self.broadcast_object(spec)
        result, digest = {}, hashlib.sha256()
        for name, shape, dtype in spec:
            if self.rank == self.leader:
                value = state[name].detach().cpu().contiguous()
            else:
                value = torch.empty(shape, dtype=getattr(torch, dtype))
            raw = value.view(torch.uint8) if value.numel() else value.reshape(0).view(torch.uint8)
            dist.broadcast(raw, src=self.leader)
            digest.update(name.encode())
            digest.update(memoryview(raw.numpy()))
            result[name] = value
        self.assert_same(digest.hexdigest(), "promoted weights")
        return result

    def join_grad_sync(self):
        """Make the current stream wait for any in-flight peer exchange."""
        if self._grad_sync is not None:
            self._grad_sync.wait()

    def check_grad_sync(self):
        if self._grad_sync is not None:
            self._grad_sync.check()

    def grad_sync(self):
        """Lazily created peer-memory gradient exchange (NCCL, one node, world > 1)."""
        if self._grad_sync is None and self.world > 1 and self.backend == "nccl" and self.single_node:
            from .grad_sync import PeerGradExchange
            self._grad_sync = PeerGradExchange(self)
        return self._grad_sync
