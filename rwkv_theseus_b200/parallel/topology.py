"""Process topology: a Gloo world group for control, one student group for data.

Contract (reference ``theseus/distributed.py:11-111``): the job is launched by
torchrun with the same number of ranks on every node; each local rank drives
one GPU (or the CPU in Gloo test mode); a Gloo process group over all ranks
carries configuration agreement, barriers and object broadcasts; the student
group (NCCL on GPUs, Gloo in CPU tests) carries gradients and metric sums and is
warmed with a one-element all-reduce before any large allocation. Ranks that
disagree on the launch shape, or two ranks on one GPU, are rejected.

Structure here: ``LaunchEnv`` reads and checks the torchrun variables,
``RankFacts`` is what every rank reports about itself, and ``Topology`` holds
the groups. Weight broadcasts pack every tensor into one byte buffer (one
collective) and finish with a digest agreement. The topology also owns the
one-node peer-memory gradient exchange (``parallel.grad_sync``), created on
first use when the student group is NCCL and every rank sits on one node.
"""
import hashlib
import json
import os
import socket
from dataclasses import dataclass
from datetime import timedelta
from typing import NamedTuple, Optional

import torch
import torch.distributed as dist


def _read_env(name, fallback=None):
    raw = os.environ.get(name)
    if raw is not None:
        return int(raw)
    if fallback is None:
        raise KeyError(f"{name} is not set; launch with torchrun")
    return fallback


@dataclass(frozen=True)
class LaunchEnv:
    rank: int
    world: int
    local_rank: int
    local_world: int

    @classmethod
    def from_environment(cls):
        world = _read_env("WORLD_SIZE")
        env = cls(_read_env("RANK"), world, _read_env("LOCAL_RANK"), _read_env("LOCAL_WORLD_SIZE", world))
        uniform = env.world >= 1 and env.local_world >= 1 and env.world % env.local_world == 0
        if not uniform or env.local_rank != env.rank % env.local_world:
            raise ValueError("Use uniform torchrun rank allocation")
        return env


class RankFacts(NamedTuple):
    local_world: int
    backend: str
    host: str
    gpu: Optional[str]


def _check_reports(mine, reports):
    """Every rank launched the same way; no GPU is driven by two ranks. Returns whether all share one host."""
    if any((r.local_world, r.backend) != (mine.local_world, mine.backend) for r in reports):
        raise ValueError("Inconsistent rank configuration")
    gpus = [(r.host, r.gpu) for r in reports if r.gpu is not None]
    if len(set(gpus)) != len(gpus):
        raise ValueError("Multiple ranks share a GPU")
    return len({r.host for r in reports}) == 1


def _digest(value):
    return hashlib.sha256(json.dumps(value, sort_keys=True, default=str).encode()).hexdigest()


def _select_device(backend, env):
    if backend == "gloo":
        return torch.device("cpu")
    if backend != "nccl":
        raise ValueError(backend)
    if not torch.cuda.is_available() or torch.cuda.device_count() < env.local_world:
        raise RuntimeError("Need one visible GPU per local rank")
    torch.cuda.set_device(env.local_rank)
    if not torch.cuda.is_bf16_supported():
        raise RuntimeError("BF16-capable GPUs are required")
    return torch.device("cuda", env.local_rank)


class Topology:
    def __init__(self, backend="nccl", timeout_minutes=60):
        env = LaunchEnv.from_environment()
        self.rank, self.world = env.rank, env.world
        self.local_rank, self.local_world = env.local_rank, env.local_world
        self.backend = backend
        self.device = _select_device(backend, env)
        self.timeout = timedelta(minutes=timeout_minutes)
        if not dist.is_initialized():
            dist.init_process_group("gloo", timeout=self.timeout)
        gpu = str(torch.cuda.get_device_properties(self.device).uuid) if self.device.type == "cuda" else None
        mine = RankFacts(env.local_world, backend, socket.gethostname(), gpu)
        self.single_node = _check_reports(mine, [RankFacts(*r) for r in self._gather(tuple(mine))])
        self.leader = 0
        self.students = list(range(self.world))
        self.groups = []
        self.tracker = None
        self._grad_sync = None
        self.student_group = self._open_group(self.students)

    # ---------------------------------------------------------------- groups
    def _gather(self, value):
        slots = [None] * self.world
        dist.all_gather_object(slots, value)
        return slots

    def _open_group(self, members):
        """New group of `members` on the data backend, proven with a one-element all-reduce before returning."""
        group = dist.new_group(members, backend=self.backend, timeout=self.timeout)
        self.groups.append(group)
        if self.rank in members:
            probe = torch.ones(1, device=self.device)
            dist.all_reduce(probe, group=group)
            self.synchronize()
            if probe.item() != len(members):
                raise RuntimeError("Process group warm-up failed")
        dist.barrier()  # the Gloo world group: also ranks outside `members`
        return group

    def synchronize(self):
        """Wait for this rank's device work (nothing to wait for on CPU ranks)."""
        if self.device.type != "cuda":
            return
        torch.cuda.synchronize(self.device)

    def barrier(self):
        """Device work finished here, then every rank of the Gloo world meets."""
        self.synchronize()
        dist.barrier()

    def close(self):
        """Collective shutdown: the peer exchange's mappings are released before the process groups."""
        self.barrier()
        exchange = self._grad_sync
        self._grad_sync = None
        if exchange:
            exchange.close()
        dist.destroy_process_group()

    # ---------------------------------------------------------------- control plane
    def assert_same(self, value, label):
        """Raise on every rank unless all ranks hold an equal (JSON-serialisable) `value`."""
        digests = self._gather(_digest(value))
        if len(set(digests)) > 1:
            raise ValueError(f"Ranks disagree on {label}: {digests}")

    def broadcast_object(self, value, source=None):
        """`source`'s (default: the leader's) picklable `value` on every rank."""
        self.synchronize()
        holder = [value if self.rank == (self.leader if source is None else source) else None]
        dist.broadcast_object_list(holder, src=self.leader if source is None else source)
        (received,) = holder
        return received

    def broadcast_weights(self, state):
        """The leader's tensors on every rank (CPU), as one packed byte buffer, followed by a digest check."""
        self.barrier()
        layout = None
        if self.rank == self.leader:
            layout, offset = [], 0
            for name in sorted(state):
                tensor = state[name]
                nbytes = tensor.numel() * tensor.element_size()
                layout.append((name, tuple(tensor.shape), str(tensor.dtype).removeprefix("torch."), offset, nbytes))
                offset += nbytes
        layout = self.broadcast_object(layout)
        total = layout[-1][3] + layout[-1][4] if layout else 0
        packed = torch.empty(total, dtype=torch.uint8)
        if self.rank == self.leader:
            for name, _, _, offset, nbytes in layout:
                if nbytes:
                    packed[offset:offset + nbytes] = state[name].detach().cpu().contiguous().reshape(-1).view(torch.uint8)
        if total:
            dist.broadcast(packed, src=self.leader)
        out = {}
        for name, shape, dtype, offset, nbytes in layout:
            out[name] = packed[offset:offset + nbytes].clone().view(getattr(torch, dtype)).reshape(shape)
        check = hashlib.sha256(json.dumps([entry[:3] for entry in layout]).encode())
        check.update(memoryview(packed.numpy()))
        self.assert_same(check.hexdigest(), "promoted weights")
        return out

    # ---------------------------------------------------------------- data plane
    def student_sum(self, tensor):
        """In-place sum over the student group (issued on the current stream)."""
        if self.world > 1:
            dist.all_reduce(tensor, group=self.student_group)
        return tensor

    def grad_sync(self):
        """The peer-memory gradient exchange, created on first use (NCCL, one node, more than one rank)."""
        if self._grad_sync is None and self.world > 1 and self.backend == "nccl" and self.single_node:
            from .grad_sync import PeerGradExchange
            self._grad_sync = PeerGradExchange(self)
        return self._grad_sync

    def join_grad_sync(self):
        """Make the current stream wait for every exchange issued so far."""
        if self._grad_sync is not None:
            self._grad_sync.wait()

    def check_grad_sync(self):
        """Raise if a device-side wait of an exchange ran out."""
        if self._grad_sync is not None:
            self._grad_sync.check()
