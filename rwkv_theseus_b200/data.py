"""Token-manifest v1 readers with resumable cursors.

File contract (the reference's, ``README.md:105-139``): ``manifest.json`` holds
``{"format": 1, "vocab_size", "sources": [{"tokens", "offsets", "weight",
"tokens_sha256", "offsets_sha256", ...}]}``; ``tokens`` is raw little-endian
uint32 and ``offsets`` an int64 ``.npy`` of N+1 strictly increasing document
boundaries from 0 to len(tokens).

Which tokens a run reads is also a contract (runs and checkpoints move between
this project and the reference, ``theseus/data.py:19-222``), so the sampling
steps below are fixed:

* sampled mode (``TokenStream``, also every validation reader): window ``w`` of
  rank ``r`` out of ``R`` draws from ``default_rng(SeedSequence([seed, w*R + r]))``
  a source by weight, then a document uniformly, then a start for a span that
  is a whole number of chunks (at most ``context_tokens``; shorter documents
  are taken whole);
* epoch mode (``EpochTokenStream``): every document is cut into windows of
  ``context_tokens`` (source, document, position order); the table is shuffled
  once by ``default_rng(seed)`` and rank ``r`` takes rows ``r::R``;
* lanes (``BatchedEpochTokenStream``, ``micro_batch_size`` > 1): the rank's
  windows are grouped by length in reading order, a group is emitted whenever
  ``micro_batch_size`` windows of one length have collected, and the leftover
  partial groups follow in first-seen length order.

The corpus (``Corpus``) is shared; each reader only decides which window comes
next and cuts it into chunks. Batches are CPU int64 tensors.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import torch

def sha256_of_file(path):
    """SHA-256 of a file's bytes, read in 8 MiB blocks."""
    hasher = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(8 << 20), b""):
            hasher.update(block)
    return hasher.hexdigest()


# Version of the window-sampling steps, stored in every reader cursor (a cursor of another version is refused).
SAMPLER_VERSION = 2


class Corpus:
    """The validated sources of one manifest: memory-mapped tokens, document offsets, normalised weights."""

    def __init__(self, manifest):
        self.path = Path(manifest).resolve()
        self.spec = json.loads(self.path.read_text())
        if self.spec.get("format") != 1:
            raise ValueError("Unsupported token manifest")
        if not self.spec["sources"]:
            raise ValueError("Manifest must contain at least one source")
        self.fingerprint = sha256_of_file(self.path)
        self.tokens, self.offsets, weights = [], [], []
        for entry in self.spec["sources"]:
            tokens = np.memmap(self.path.parent / entry["tokens"], dtype="<u4", mode="r")
            offsets = np.load(self.path.parent / entry["offsets"], mmap_mode="r")
            well_formed = (len(offsets) >= 2 and offsets[0] == 0 and offsets[-1] == len(tokens)
                           and bool(np.all(np.diff(offsets) > 0)))
            if not well_formed:
                raise ValueError("Invalid or empty document offsets")
            if not (np.isfinite(entry["weight"]) and entry["weight"] > 0):
                raise ValueError("Mixture weights must be positive")
            self.tokens.append(tokens)
            self.offsets.append(offsets)
            weights.append(float(entry["weight"]))
        self.weights = np.asarray(weights) / np.sum(weights)

    def span(self, source, begin, end):
        return self.tokens[int(source)][int(begin):int(end)]

    def total_tokens(self):
        return int(sum(len(t) for t in self.tokens))

    def window_table(self, context_tokens):
        """Every (source, begin, end) window of at most `context_tokens` tokens inside one document, in
        source, document and position order."""
        tables = []
        for source, offsets in enumerate(self.offsets):
            bounds = np.asarray(offsets, dtype=np.int64)
            doc_len = bounds[1:] - bounds[:-1]
            pieces = -(-doc_len // context_tokens)                     # windows per document
            owner = np.repeat(np.arange(len(doc_len)), pieces)         # document of each window
            index_in_doc = np.arange(len(owner)) - np.repeat(np.cumsum(pieces) - pieces, pieces)
            begin = bounds[owner] + index_in_doc * context_tokens
            end = np.minimum(begin + context_tokens, bounds[owner + 1])
            tables.append(np.stack([np.full_like(begin, source), begin, end], axis=1))
        return np.concatenate(tables).astype(np.int64, copy=False)


def _as_ids(array):
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.int64))


def _chunk_count(lengths, chunk_tokens):
    return -(-np.asarray(lengths, dtype=np.int64) // chunk_tokens)


class TokenStream:
    """Sampled windows (mixture by source weight), cut into chunks; never exhausted."""

    def __init__(self, manifest, pair_id, pairs, chunk_tokens, context_tokens, seed=42):
        self.corpus = Corpus(manifest)
        self.path, self.manifest, self.fingerprint = self.corpus.path, self.corpus.spec, self.corpus.fingerprint
        if chunk_tokens < 1 or context_tokens < chunk_tokens:
            raise ValueError("Require context_tokens >= chunk_tokens >= 1")
        self.pair_id, self.pairs, self.seed = pair_id, pairs, seed
        self.chunk_tokens, self.context_tokens = chunk_tokens, context_tokens
        self.window = self.offset = self.chunks = 0   # cursor: window index, position in it, chunks emitted
        self._tokens = None                           # the current window's tokens

    # which window comes next ------------------------------------------------------------
    def _stream_id(self):
        return self.window * self.pairs + self.pair_id

    def _draw_window(self):
        draw = np.random.default_rng(np.random.SeedSequence([self.seed, self._stream_id()]))
        source = int(draw.choice(len(self.corpus.tokens), p=self.corpus.weights))
        offsets = self.corpus.offsets[source]
        doc = int(draw.integers(len(offsets) - 1))
        doc_begin, doc_end = int(offsets[doc]), int(offsets[doc + 1])
        size = doc_end - doc_begin
        take = size if size < self.chunk_tokens else min(size, self.context_tokens) // self.chunk_tokens * \
            self.chunk_tokens
        begin = doc_begin + int(draw.integers(size - take + 1))
        return self.corpus.span(source, begin, begin + take)

    # chunking ------------------------------------------------------------------------------
    def next(self):
        if self._tokens is None:
            self._tokens = self._draw_window()
        stop = min(len(self._tokens), self.offset + self.chunk_tokens)
        batch = {"ids": _as_ids(self._tokens[self.offset:stop])[None], "reset": self.offset == 0,
                 "stream": self._stream_id(), "chunk": self.chunks, "position": self.offset}
        self.chunks += 1
        if stop < len(self._tokens):
            self.offset = stop
        else:
            self.window, self.offset, self._tokens = self.window + 1, 0, None
        return batch

    # resume ---------------------------------------------------------------------------------
    _CURSOR = ("window", "offset", "chunks")

    def _identity(self):
        return {"fingerprint": self.fingerprint, "pair_id": self.pair_id, "pairs": self.pairs, "seed": self.seed,
                "chunk_tokens": self.chunk_tokens, "context_tokens": self.context_tokens,
                "sampler_version": SAMPLER_VERSION}

    def state_dict(self):
        return {name: getattr(self, name) for name in self._CURSOR} | self._identity()

    def _check_identity(self, state):
        for key, value in self._identity().items():
            if key not in state or state[key] != value:
                raise ValueError(f"Reader resume mismatch: {key}")

    def load_state_dict(self, state):
        self._check_identity(state)
        for name in self._CURSOR:
            setattr(self, name, state[name])
        self._tokens = None


class EpochTokenStream(TokenStream):
    """Every token of the corpus exactly once: this rank's share of one shuffled window table."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        table = self.corpus.window_table(self.context_tokens)
        np.random.default_rng(self.seed).shuffle(table)
        self._table = table
        chunks = _chunk_count(table[:, 2] - table[:, 1], self.chunk_tokens)
        self.rank_chunks = [int(chunks[rank::self.pairs].sum()) for rank in range(self.pairs)]
        self.total_tokens = self.corpus.total_tokens()
        self.windows = table[self.pair_id::self.pairs].copy()
        self.consumed_tokens = 0

    MODE = "epoch_v1"  # reader_mode recorded in (and required of) a checkpoint cursor

    @property
    def exhausted(self):
        return not self.window < len(self.windows)

    def _draw_window(self):
        if self.exhausted:
            raise StopIteration
        return self.corpus.span(*self.windows[self.window])

    def next(self):
        """The next chunk of this rank's share, or None once every window was read."""
        batch = None if self.exhausted else super().next()
        if batch is not None:
            self.consumed_tokens += batch["ids"].numel()
        return batch

    def state_dict(self):
        cursor = super().state_dict()
        cursor.update(reader_mode=self.MODE, consumed_tokens=self.consumed_tokens)
        return cursor

    def load_state_dict(self, state):
        mode = state.get("reader_mode")
        if mode != self.MODE:
            raise ValueError(f"Reader mode {mode!r} cannot resume an exhaustive epoch ({self.MODE})")
        super().load_state_dict(state)
        self.consumed_tokens = state["consumed_tokens"]


def pack_lanes(windows, lanes):
    """Groups of `lanes` equal-length windows in reading order; leftovers last, in first-seen length order."""
    waiting, groups = {}, []
    for row in windows:
        bucket = waiting.setdefault(int(row[2] - row[1]), [])
        bucket.append(row)
        if len(bucket) == lanes:
            groups.append(np.stack(bucket).astype(np.int64))
            bucket.clear()
    groups.extend(np.stack(bucket).astype(np.int64) for bucket in waiting.values() if bucket)
    return groups


class BatchedEpochTokenStream(EpochTokenStream):
    """Epoch mode with `micro_batch_size` independent lanes of equal-length windows (no padding: every lane starts
    and ends at the same positions, so caches and recurrent states reset per group)."""

    def __init__(self, *args, micro_batch_size, **kwargs):
        self.micro_batch_size = int(micro_batch_size)
        if self.micro_batch_size <= 1:
            raise ValueError(f"lane packing needs micro_batch_size >= 2, got {micro_batch_size}")
        super().__init__(*args, **kwargs)
        self.groups = pack_lanes(self.windows, micro_batch_size)
        self.rank_chunks = [self._packed_chunks(self._table[rank::self.pairs]) for rank in range(self.pairs)]
        del self.windows, self._table
        self.group = self.offset = 0

    def _packed_chunks(self, windows):
        lengths, count = np.unique(windows[:, 2] - windows[:, 1], return_counts=True)
        groups = -(-count // self.micro_batch_size)
        return int((groups * _chunk_count(lengths, self.chunk_tokens)).sum())

    @property
    def exhausted(self):
        return not self.group < len(self.groups)

    def next(self):
        """The next chunk of the current lane group ([lanes, tokens]), or None once every group was read."""
        if self.exhausted:
            return None
        rows = self.groups[self.group]
        length = int(rows[0, 2] - rows[0, 1])
        stop = min(length, self.offset + self.chunk_tokens)
        ids = _as_ids(np.stack([self.corpus.span(s, b + self.offset, b + stop) for s, b, _ in rows]))
        batch = {"ids": ids, "reset": self.offset == 0, "position": self.offset, "group": self.group}
        self.consumed_tokens += ids.numel()
        if stop < length:
            self.offset = stop
        else:
            self.group, self.offset = self.group + 1, 0
        return batch

    _CURSOR = ("group", "offset", "consumed_tokens")

    def _identity(self):
        return super()._identity() | {"reader_mode": "batched_epoch_v1", "micro_batch_size": self.micro_batch_size}

    def state_dict(self):
        return self._identity() | {name: getattr(self, name) for name in self._CURSOR}

    def load_state_dict(self, state):
        for key, value in self._identity().items():
            if state.get(key) != value:
                raise ValueError(f"Reader resume mismatch: {key}")
        for name in self._CURSOR:
            setattr(self, name, state[name])


def reader_for(cfg, topo, validation=False):
    """The reader a run uses (reference ``theseus/validation.py:13-22``): sampled windows for validation and for
    ``training_mode: sampled``, the epoch reader otherwise (lane-packed when ``micro_batch_size`` > 1)."""
    manifest = cfg["validation_manifest" if validation else "train_manifest"]
    common = (manifest, topo.rank, topo.world, cfg["chunk_tokens"], cfg["context_tokens"], cfg["seed"])
    if validation or cfg.get("training_mode", "sampled") != "epoch":
        return TokenStream(*common)
    if cfg.get("micro_batch_size", 1) > 1:
        return BatchedEpochTokenStream(*common, micro_batch_size=cfg["micro_batch_size"])
    return EpochTokenStream(*common)
