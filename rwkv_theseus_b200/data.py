"""Token-manifest v1 readers with resumable cursors.

File contract (unchanged from the reference, ``README.md:105-139``): a
``manifest.json`` with ``{"format": 1, "vocab_size", "sources": [{"tokens",
"offsets", "weight", "tokens_sha256", "offsets_sha256", ...}]}``; ``tokens`` is
raw little-endian uint32, ``offsets`` an int64 ``.npy`` of N+1 strictly
increasing document boundaries from 0 to len(tokens).

The three readers reproduce the reference's sampling semantics exactly
(``theseus/data.py:19-222``) so that runs and checkpoints are interchangeable:

* ``TokenStream`` (``training_mode: sampled`` and validation): each window is
  drawn with ``default_rng(SeedSequence([seed, window * pairs + pair_id]))``:
  source by weight, document uniformly, then a whole number of chunks (at most
  ``context_tokens``) at a random start.
* ``EpochTokenStream``: every token exactly once. Documents are cut into
  windows of ``context_tokens``; the window list is shuffled once with
  ``default_rng(seed)`` and rank r takes entries ``r::world``.
* ``BatchedEpochTokenStream``: the rank's windows are packed into groups of
  ``micro_batch_size`` equal-length windows (independent lanes sharing the
  same positions); leftovers form smaller groups.

Batches are plain CPU int64 tensors; the trainer stages them through one
persistent pinned buffer so each step's host-to-device copy is asynchronous.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import torch

SAMPLER_VERSION = 2


def digest_file(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            block = f.read(8 << 20)
            if not block:
                break
            h.update(block)
    return h.hexdigest()


def _ids_tensor(values):
    return torch.from_numpy(np.ascontiguousarray(values, dtype=np.int64))


class TokenStream:
    def __init__(self, manifest, pair_id, pairs, chunk_tokens, context_tokens, seed=42):
        self.path = Path(manifest).resolve()
        self.manifest = json.loads(self.path.read_text())
        if self.manifest.get("format") != 1:
            raise ValueError("Unsupported token manifest")
        if chunk_tokens < 1 or context_tokens < chunk_tokens:
            raise ValueError("Require context_tokens >= chunk_tokens >= 1")
        self.fingerprint = digest_file(self.path)
        self.pair_id, self.pairs = pair_id, pairs
        self.chunk_tokens, self.context_tokens, self.seed = chunk_tokens, context_tokens, seed
        if not self.manifest["sources"]:
            raise ValueError("Manifest must contain at least one source")
        self.sources, weights = [], []
        for entry in self.manifest["sources"]:
            tokens = np.memmap(self.path.parent / entry["tokens"], dtype="<u4", mode="r")
            offsets = np.load(self.path.parent / entry["offsets"], mmap_mode="r")
            bad = (len(offsets) < 2 or offsets[0] != 0 or offsets[-1] != len(tokens)
                   or bool(np.any(np.diff(offsets) <= 0)))
            if bad:
                raise ValueError("Invalid or empty document offsets")
            if not np.isfinite(entry["weight"]) or entry["weight"] <= 0:
                raise ValueError("Mixture weights must be positive")
            self.sources.append((tokens, offsets))
            weights.append(entry["weight"])
        self.weights = np.asarray(weights, dtype=np.float64)
        self.weights /= self.weights.sum()
        self.window = self.offset = self.chunks = 0
        self._current = None

    def _window(self):
        stream = self.window * self.pairs + self.pair_id
        rng = np.random.default_rng(np.random.SeedSequence([self.seed, stream]))
        tokens, offsets = self.sources[int(rng.choice(len(self.sources), p=self.weights))]
        doc = int(rng.integers(len(offsets) - 1))
        begin, finish = int(offsets[doc]), int(offsets[doc + 1])
        available = finish - begin
        if available >= self.chunk_tokens:
            length = min(available, self.context_tokens) // self.chunk_tokens * self.chunk_tokens
        else:
            length = available
        begin += int(rng.integers(available - length + 1))
        return tokens[begin:begin + length]

    def next(self):
        if self._current is None:
            self._current = self._window()
        stop = min(len(self._current), self.offset + self.chunk_tokens)
        ids = _ids_tensor(self._current[self.offset:stop])[None]
        batch = {"ids": ids, "reset": self.offset == 0, "stream": self.window * self.pairs + self.pair_id,
                 "chunk": self.chunks, "position": self.offset}
        self.offset = stop
        self.chunks += 1
        if stop == len(self._current):
            self.window += 1
            self.offset = 0
            self._current = None
        return batch

    def state_dict(self):
        return {"window": self.window, "offset": self.offset, "chunks": self.chunks,
                "fingerprint": self.fingerprint, "pair_id": self.pair_id, "pairs": self.pairs,
                "seed": self.seed, "chunk_tokens": self.chunk_tokens,
                "context_tokens": self.context_tokens, "sampler_version": SAMPLER_VERSION}

    def load_state_dict(self, state):
        own = self.state_dict()
        for key in own.keys() - {"window", "offset", "chunks"}:
            if key not in state or own[key] != state[key]:
                raise ValueError(f"Reader resume mismatch: {key}")
        self.window, self.offset, self.chunks = state["window"], state["offset"], state["chunks"]
        self._current = None


def _epoch_windows(sources, context_tokens):
    """All (source, start, end) windows of at most ``context_tokens`` inside documents."""
    parts = []
    for source, (_, offsets) in enumerate(sources):
        offsets = np.asarray(offsets, dtype=np.int64)
        lengths = np.diff(offsets)
        per_doc = (lengths + context_tokens - 1) // context_tokens
        doc = np.repeat(np.arange(len(per_doc)), per_doc)
        first = np.repeat(np.cumsum(per_doc) - per_doc, per_doc)
        starts = offsets[doc] + (np.arange(len(doc)) - first) * context_tokens
        ends = np.minimum(starts + context_tokens, offsets[doc + 1])
        parts.append(np.column_stack((np.full(len(doc), source), starts, ends)))
    return np.concatenate(parts).astype(np.int64, copy=False)


class EpochTokenStream(TokenStream):
    """Visit every token exactly once; ranks take disjoint shuffled windows."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        windows = _epoch_windows(self.sources, self.context_tokens)
        np.random.default_rng(self.seed).shuffle(windows)
        self._all_windows = windows if getattr(self, "micro_batch_size", 1) > 1 else None
        costs = (windows[:, 2] - windows[:, 1] + self.chunk_tokens - 1) // self.chunk_tokens
        self.rank_chunks = [int(costs[r::self.pairs].sum()) for r in range(self.pairs)]
        self.total_tokens = sum(len(tokens) for tokens, _ in self.sources)
        self.windows = windows[self.pair_id::self.pairs].copy()
        self.consumed_tokens = 0

    def _window(self):
        if self.exhausted:
            raise StopIteration
        source, begin, finish = self.windows[self.window]
        return self.sources[source][0][begin:finish]

    @property
    def exhausted(self):
        return self.window >= len(self.windows)

    def next(self):
        if self.exhausted:
            return None
        batch = super().next()
        self.consumed_tokens += batch["ids"].numel()
        return batch

    def state_dict(self):
        return super().state_dict() | {"reader_mode": "epoch_v1", "consumed_tokens": self.consumed_tokens}

    def load_state_dict(self, state):
        if state.get("reader_mode") != "epoch_v1":
            raise ValueError("A sampled reader checkpoint cannot resume an exhaustive epoch")
        self.consumed_tokens = state["consumed_tokens"]
        super().load_state_dict(state)


class BatchedEpochTokenStream(EpochTokenStream):
    """Equal-length windows packed into ``micro_batch_size`` independent lanes."""

    def __init__(self, *args, micro_batch_size, **kwargs):
        if micro_batch_size < 2:
            raise ValueError("Batched reader requires micro_batch_size >= 2")
        self.micro_batch_size = micro_batch_size
        super().__init__(*args, **kwargs)
        self.groups = self._pack(self.windows)
        self.rank_chunks = []
        for rank in range(self.pairs):
            mine = self._all_windows[rank::self.pairs]
            lengths, counts = np.unique(mine[:, 2] - mine[:, 1], return_counts=True)
            groups_per_length = (counts + micro_batch_size - 1) // micro_batch_size
            chunks_per_group = (lengths + self.chunk_tokens - 1) // self.chunk_tokens
            self.rank_chunks.append(int((groups_per_length * chunks_per_group).sum()))
        del self.windows, self._all_windows
        self.group = self.offset = 0

    def _pack(self, windows):
        pending, groups = {}, []
        for row in windows:
            bucket = pending.setdefault(int(row[2] - row[1]), [])
            bucket.append(row)
            if len(bucket) == self.micro_batch_size:
                groups.append(np.asarray(bucket, dtype=np.int64))
                bucket.clear()
        groups.extend(np.asarray(b, dtype=np.int64) for b in pending.values() if b)
        return groups

    @property
    def exhausted(self):
        return self.group >= len(self.groups)

    def next(self):
        if self.exhausted:
            return None
        group = self.groups[self.group]
        length = int(group[0, 2] - group[0, 1])
        stop = min(length, self.offset + self.chunk_tokens)
        rows = [np.asarray(self.sources[int(s)][0][int(b) + self.offset:int(b) + stop], dtype=np.int64)
                for s, b, _ in group]
        ids = _ids_tensor(np.stack(rows))
        batch = {"ids": ids, "reset": self.offset == 0, "position": self.offset, "group": self.group}
        self.consumed_tokens += ids.numel()
        self.offset = stop
        if stop == length:
            self.group += 1
            self.offset = 0
        return batch

    def state_dict(self):
        return {"reader_mode": "batched_epoch_v1", "fingerprint": self.fingerprint,
                "pair_id": self.pair_id, "pairs": self.pairs, "seed": self.seed,
                "chunk_tokens": self.chunk_tokens, "context_tokens": self.context_tokens,
                "sampler_version": SAMPLER_VERSION, "micro_batch_size": self.micro_batch_size,
                "group": self.group, "offset": self.offset, "consumed_tokens": self.consumed_tokens}

    def load_state_dict(self, state):
        own = self.state_dict()
        for key in own.keys() - {"group", "offset", "consumed_tokens"}:
            if own[key] != state.get(key):
                raise ValueError(f"Reader resume mismatch: {key}")
        self.group, self.offset = state["group"], state["offset"]
        self.consumed_tokens = state["consumed_tokens"]


def reader_for(cfg, topo, validation=False):
    """Reader class selection (reference ``theseus/validation.py:13-22``)."""
    if validation or cfg.get("training_mode", "sampled") != "epoch":
        cls, extra = TokenStream, {}
    elif cfg.get("micro_batch_size", 1) > 1:
        cls, extra = BatchedEpochTokenStream, {"micro_batch_size": cfg["micro_batch_size"]}
    else:
        cls, extra = EpochTokenStream, {}
    manifest = cfg["validation_manifest" if validation else "train_manifest"]
    return cls(manifest, topo.rank, topo.world, cfg["chunk_tokens"], cfg["context_tokens"], cfg["seed"], **extra)
