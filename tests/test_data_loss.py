"""Manifest readers and distillation statistics.

The readers' token order is a cross-project contract, so the sampled reader is checked against an independent
restatement of its window rule, and the epoch readers against coverage (every token exactly once over all ranks),
their chunk accounting and lossless resume from any cursor."""
import json

import numpy as np
import pytest
import torch

from fixtures import write_dataset
from rwkv_theseus_b200.config import steps_for
from rwkv_theseus_b200.data import BatchedEpochTokenStream, EpochTokenStream, TokenStream, pack_lanes
from rwkv_theseus_b200.losses import metrics, statistics


def two_source_manifest(path):
    """Two sources (weights 1 and 3) of documents with distinct token ranges."""
    path.mkdir(parents=True, exist_ok=True)
    sources = []
    for name, lengths, base in (("a", [5, 12, 2, 9], 0), ("b", [20, 3, 7], 1000)):
        tokens = np.arange(base, base + sum(lengths), dtype=np.uint32)
        tokens.astype("<u4").tofile(path / f"{name}.bin")
        np.save(path / f"{name}.npy", np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64))
        sources.append({"tokens": f"{name}.bin", "offsets": f"{name}.npy", "weight": 1 if name == "a" else 3})
    (path / "manifest.json").write_text(json.dumps({"format": 1, "vocab_size": 2048, "sources": sources}))
    return path / "manifest.json", [np.arange(0, 28), np.arange(1000, 1030)], [[0, 5, 17, 19, 28], [0, 20, 23, 30]]


def expected_window(seed, stream, tokens, offsets, weights, chunk, context):
    """The sampled-window rule, restated: source by weight, document uniformly, then a start for a span that is a
    whole number of chunks (documents shorter than one chunk are taken whole)."""
    rng = np.random.default_rng(np.random.SeedSequence([seed, stream]))
    source = int(rng.choice(len(tokens), p=np.asarray(weights) / np.sum(weights)))
    bounds = offsets[source]
    doc = int(rng.integers(len(bounds) - 1))
    size = bounds[doc + 1] - bounds[doc]
    take = size if size < chunk else min(size, context) // chunk * chunk
    begin = bounds[doc] + int(rng.integers(size - take + 1))
    return tokens[source][begin:begin + take]


@pytest.mark.parametrize("rank,ranks", [(0, 1), (1, 3)])
def test_sampled_reader_matches_the_window_rule(tmp_path, rank, ranks):
    manifest, tokens, offsets = two_source_manifest(tmp_path)
    reader = TokenStream(manifest, rank, ranks, chunk_tokens=4, context_tokens=10, seed=5)
    for window in range(12):
        want = expected_window(5, window * ranks + rank, tokens, offsets, [1, 3], 4, 10)
        got = []
        while True:
            batch = reader.next()
            assert batch["stream"] == window * ranks + rank and batch["position"] == len(got)
            assert batch["reset"] == (len(got) == 0) and batch["ids"].shape[0] == 1
            got.extend(batch["ids"][0].tolist())
            if len(got) == len(want):
                break
        assert got == want.tolist()


def test_sampled_reader_resumes_mid_window_and_rejects_other_settings(tmp_path):
    manifest, _, _ = two_source_manifest(tmp_path)
    reader = TokenStream(manifest, 0, 2, 3, 9, seed=1)
    for _ in range(5):
        reader.next()
    saved = reader.state_dict()
    ahead = [reader.next() for _ in range(8)]
    clone = TokenStream(manifest, 0, 2, 3, 9, seed=1)
    clone.load_state_dict(saved)
    for batch in ahead:
        other = clone.next()
        assert torch.equal(other.pop("ids"), batch.pop("ids")) and other == batch
    for changed in (dict(seed=2), dict(chunk_tokens=4)):
        args = dict(chunk_tokens=3, context_tokens=9, seed=1) | changed
        with pytest.raises(ValueError, match="Reader resume mismatch"):
            TokenStream(manifest, 0, 2, **args).load_state_dict(saved)


def drain(reader):
    out = []
    while (batch := reader.next()) is not None:
        out.append(batch)
    return out


@pytest.mark.parametrize("ranks,chunk,context", [(1, 4, 7), (3, 2, 5), (4, 3, 30)])
def test_epoch_reader_covers_every_token_once(tmp_path, ranks, chunk, context):
    manifest, tokens, _ = two_source_manifest(tmp_path)
    seen = []
    for rank in range(ranks):
        reader = EpochTokenStream(manifest, rank, ranks, chunk, context, seed=3)
        batches = drain(reader)
        assert reader.exhausted and reader.next() is None
        assert len(batches) == reader.rank_chunks[rank]
        for batch in batches:
            assert batch["ids"].shape[1] <= chunk and batch["position"] + batch["ids"].shape[1] <= context
            seen.extend(batch["ids"][0].tolist())
        assert reader.consumed_tokens == sum(b["ids"].numel() for b in batches)
    assert sorted(seen) == sorted(np.concatenate(tokens).tolist())


def test_epoch_reader_resume_and_mode_check(tmp_path):
    manifest, _, _ = two_source_manifest(tmp_path)
    reader = EpochTokenStream(manifest, 1, 2, 3, 8, seed=4)
    reader.next(), reader.next(), reader.next()
    state = reader.state_dict()
    rest = drain(reader)
    clone = EpochTokenStream(manifest, 1, 2, 3, 8, seed=4)
    clone.load_state_dict(state)
    assert [b["ids"].tolist() for b in drain(clone)] == [b["ids"].tolist() for b in rest]
    with pytest.raises(ValueError, match="cannot resume"):
        clone.load_state_dict(TokenStream(manifest, 1, 2, 3, 8, seed=4).state_dict())


def test_lane_packing_rule():
    rows = np.array([[0, 0, 4], [0, 10, 13], [0, 20, 24], [0, 30, 33], [0, 40, 45], [0, 50, 54]])
    groups = pack_lanes(rows, 2)
    assert [g[:, 1].tolist() for g in groups] == [[0, 20], [10, 30], [50], [40]]


@pytest.mark.parametrize("lanes", [2, 3])
def test_batched_reader_lanes_cover_tokens_and_resume(tmp_path, lanes):
    manifest, tokens, _ = two_source_manifest(tmp_path)
    seen = []
    for rank in range(2):
        reader = BatchedEpochTokenStream(manifest, rank, 2, 3, 6, seed=7, micro_batch_size=lanes)
        reader.next()
        state = reader.state_dict()
        clone = BatchedEpochTokenStream(manifest, rank, 2, 3, 6, seed=7, micro_batch_size=lanes)
        clone.load_state_dict(state)
        rest, again = drain(reader), drain(clone)
        assert [b["ids"].tolist() for b in rest] == [b["ids"].tolist() for b in again]
        fresh = drain(BatchedEpochTokenStream(manifest, rank, 2, 3, 6, seed=7, micro_batch_size=lanes))
        assert len(fresh) == reader.rank_chunks[rank]
        for batch in fresh:
            assert 1 <= batch["ids"].shape[0] <= lanes   # equal-length lanes, no padding
            seen.extend(batch["ids"].flatten().tolist())
    assert sorted(seen) == sorted(np.concatenate(tokens).tolist())


def test_fixture_dataset_windows_split_across_seven_ranks(tmp_path):
    manifest = write_dataset(tmp_path)
    collected = [t for rank in range(7)
                 for b in drain(EpochTokenStream(manifest, rank, 7, 4, 7)) for t in b["ids"][0].tolist()]
    assert sorted(collected) == list(range(37))


def test_statistics_match_their_definitions():
    torch.manual_seed(0)
    pred, target = torch.randn(2, 5, 8), torch.randn(2, 5, 8)
    mask = torch.tensor([[1., 0., 1., 1., 1.], [0., 1., 1., 0., 1.]])
    sums = statistics(pred, target, 1e-6, mask)
    nmse = ((pred - target) ** 2).mean(-1) / (target ** 2).mean(-1)
    cos = (pred * target).sum(-1) / (pred.norm(dim=-1) * target.norm(dim=-1))
    torch.testing.assert_close(sums, torch.stack([(nmse * mask).sum(), (cos * mask).sum(), mask.sum()]))
    report = metrics(sums)
    assert report["tokens"] == 7 and report["rrms"] == pytest.approx(report["nmse"] ** 0.5)
    # the epsilon floors the target energy of an all-zero target
    zero = statistics(torch.ones(1, 1, 4), torch.zeros(1, 1, 4), 0.5)
    assert zero[0].item() == pytest.approx(1 / 0.5)
    with pytest.raises(ValueError):
        metrics(torch.zeros(3))


def test_stage_budget_lists():
    assert steps_for({"stage_steps": 11}, 3) == 11
    assert steps_for({"stage_steps": [6]}, 9) == 6
    assert steps_for({"stage_steps": [2, 4, 8]}, 2) == 8
