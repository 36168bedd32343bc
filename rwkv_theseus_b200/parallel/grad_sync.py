"""Per-layer gradient exchange over NVLink peer memory (one node, 2..8 ranks).

The reference reduces each layer's gradients with an NCCL all-reduce and then
clips and steps torch AdamW over the whole layer on every rank
(``theseus/stage.py:27-44``, ``train.py:170-211``). Here the flat buffers of a
layer (fp32 gradient, fp32 parameters, bf16 weight copy) and one small signal
buffer per rank are mapped into every other rank's address space with CUDA
IPC, and ``exchange_update`` (``csrc/parallel/peer_exchange.cu``) runs the
whole update as three kernels: reduce-scatter with the squared norm (peer
loads), then clip + AdamW on this rank's 1/N shard (local), then an
all-gather that pulls the other shards of the bf16 weight copy and of the
fp32 non-decay parameters. ``fused=True`` replaces the last two by one kernel
whose update blocks raise a flag per shard slice while its pull blocks fetch
each peer's slices as their flags come up (local updates overlapping NVLink
pulls); at 2 ranks it measured 0.885 ms against 0.856 ms for the three-kernel
path on a 112M-parameter layer, so it is not the default. The global norm and
loss statistics are summed in rank order on every rank, so all ranks apply the
identical clip coefficient.

The kernels run on a side stream: the main stream continues with the next
layer's student (or the next step's teacher forward) while the exchange of
this one moves over NVLink. ``update`` returns an event per layer; the student
waits on it where its parameters are next read (its next micro-step, a
prediction, a checkpoint), so no step-wide join is needed. The fp32 masters of the four decay matrices and the Adam moments are
sharded (each rank updates only its own range; compute reads the bf16 copy);
``gather_state`` assembles them on every rank for a checkpoint or export.

Every device wait is bounded (``limit_s``); an expired wait records a status
that ``check`` turns into an exception on the host.
"""
import torch
import torch.distributed as dist

from ..ops import native

STATUS_WORD, WAITED_WORD = 24, 27
_WHAT = {1: "gradients ready", 2: "partial norm", 3: "updated shard"}


class PeerGradExchange:
    def __init__(self, topo, blocks=256, limit_s=300.0, fused=False):
        if topo.world > 8:
            raise ValueError("peer exchange supports at most 8 ranks per node")
        self.topo = topo
        self.rank, self.world = topo.rank, topo.world
        self.device = topo.device
        self.blocks = blocks
        self.fused = bool(fused)  # one update+pull kernel (per-slice flags) instead of update, then gather
        self.limit_s = float(limit_s)
        ext = native()
        self.sig = torch.zeros(ext.exchange_signal_words(), dtype=torch.int32, device=self.device)
        self.stream = torch.cuda.Stream(self.device)
        self.epoch = 0
        self._opened = {}   # (rank, peer allocation base) -> mapped base address
        self.sig_ptrs = self.share(self.sig)
        self.pending = False

    # ---------------------------------------------------------------- mapping
    def share(self, tensor):
        """Collective: every rank's address of its own ``tensor`` (peers mapped here)."""
        handle, offset = native().ipc_export(tensor)
        table = [None] * self.world
        dist.all_gather_object(table, (handle, offset, tensor.data_ptr() - offset))
        out = []
        for q, (h, off, base) in enumerate(table):
            if q == self.rank:
                out.append(tensor.data_ptr())
                continue
            key = (q, base)  # one mapping per peer allocation, however many tensors live in it
            if key not in self._opened:
                self._opened[key] = native().ipc_open(h, self.device.index)
            out.append(self._opened[key] + off)
        return out

    def register(self, student):
        """Collective (same students in the same order on every rank): map the student's buffers.

        The address tables are kept on the student object, so an exchange never runs on the addresses of
        another (possibly freed) student's buffers."""
        flat = student.flat
        student.peer_tables = (self.share(flat.grad), self.share(flat.param), self.share(student.fused.shadow))
        return student.peer_tables

    # ---------------------------------------------------------------- update
    def update(self, student, lr, step):
        """Reduce, clip, AdamW and all-gather one layer on the side stream; returns the event that marks the end of
        this layer's exchange (the caller waits on it where the layer's parameters are next read)."""
        tables = getattr(student, "peer_tables", None)
        if tables is None:
            raise RuntimeError("student buffers are not registered with the peer exchange")
        grads, params, shadows = tables
        cfg, flat = student.cfg, student.flat
        beta1, beta2 = cfg["betas"]
        self.epoch += 1
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            native().exchange_update(grads, params, shadows, self.sig_ptrs, self.rank, self.world, flat.numel,
                                     flat.exp_avg, flat.exp_avg_sq, student.stats, student.report, float(lr),
                                     float(beta1), float(beta2), float(cfg["adam_eps"]),
                                     float(cfg["weight_decay"]), float(cfg["clip_norm"]), int(step),
                                     int(student.decay_numel), self.epoch & 0xFFFFFFFF, self.limit_s, self.blocks,
                                     0 if self.fused else 1)
        done = torch.cuda.Event()
        done.record(self.stream)
        self.pending = True
        return done

    def wait(self):
        """Join the exchange stream into the current stream."""
        if self.pending:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
            self.pending = False

    def status_words(self):
        """The device status words (failure code .. waited rank) that ``check`` reads, as a tensor view."""
        return self.sig[STATUS_WORD:WAITED_WORD + 1]

    def raise_for(self, words):
        """Raise for status words read from the device (``words`` as returned by ``status_words``)."""
        if words[0]:
            raise RuntimeError(f"peer gradient exchange on rank {self.rank} timed out waiting for rank "
                               f"{words[3]}'s {_WHAT.get(words[0], 'signal')} after {self.limit_s:.0f} s")

    def check(self):
        """Raise if a device wait of any exchange so far ran out (host read of one status word)."""
        self.raise_for(self.status_words().cpu().tolist())

    # ---------------------------------------------------------------- sharded state
    def shard(self, n, rank):
        lo, hi, tail_lo, tail_hi = native().exchange_shard(n, rank, self.world)
        return [(lo, hi), (tail_lo, tail_hi)]

    def gather_state(self, student):
        """Collective: full fp32 parameters and Adam moments on every rank (each rank owns one shard)."""
        self.wait()
        flat = student.flat
        for q in range(self.world):
            for lo, hi in self.shard(flat.numel, q):
                if hi > lo:
                    for buf in (flat.param, flat.exp_avg, flat.exp_avg_sq):
                        dist.broadcast(buf[lo:hi], src=q, group=self.topo.student_group)

    def close(self):
        torch.cuda.synchronize(self.device)
        for base in self._opened.values():
            native().ipc_close(base, self.device.index)
        self._opened.clear()
