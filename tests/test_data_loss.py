import torch

from fixtures import write_dataset
from rwkv_theseus_b200.config import steps_for
from rwkv_theseus_b200.data import BatchedEpochTokenStream, EpochTokenStream, TokenStream
from rwkv_theseus_b200.losses import metrics, statistics


def test_reader_resume_and_replay(tmp_path):
    manifest = write_dataset(tmp_path)
    a = TokenStream(manifest, 0, 2, 3, 9)
    first = a.next()
    saved = a.state_dict()
    expected = [a.next() for _ in range(10)]
    b = TokenStream(manifest, 0, 2, 3, 9)
    b.load_state_dict(saved)
    for batch in expected:
        actual = b.next()
        torch.testing.assert_close(actual.pop("ids"), batch.pop("ids"))
        assert actual == batch
    torch.testing.assert_close(first["ids"], TokenStream(manifest, 0, 2, 3, 9).next()["ids"])


def test_sampler_avoids_short_tails_for_documents_at_least_one_chunk(tmp_path):
    manifest = write_dataset(tmp_path)
    stream = TokenStream(manifest, 0, 1, chunk_tokens=3, context_tokens=9, seed=9)
    for _ in range(40):
        assert stream.next()["ids"].shape[1] == 3


def test_token_weighted_loss_and_mask():
    target = torch.tensor([[[1., 1.], [10., 10.], [0., 0.]]])
    pred = torch.tensor([[[2., 2.], [0., 0.], [100., 100.]]])
    result = metrics(statistics(pred, target, mask=torch.tensor([[1., 1., 0.]])))
    assert result["nmse"] == 1 and result["rrms"] == 1 and result["tokens"] == 2


def test_singleton_stage_schedule_is_broadcast_to_all_stages():
    assert steps_for({"stage_steps": [5]}, 15) == 5
    assert steps_for({"stage_steps": [3, 7]}, 1) == 7


def test_epoch_all_tokens_once_with_tails_and_resume(tmp_path):
    manifest = write_dataset(tmp_path)
    seen = []
    for rank in range(7):
        reader = EpochTokenStream(manifest, rank, 7, 4, 7)
        first = reader.next()
        if first:
            seen.extend(first["ids"].flatten().tolist())
        resumed = EpochTokenStream(manifest, rank, 7, 4, 7)
        resumed.load_state_dict(reader.state_dict())
        while True:
            batch, other = reader.next(), resumed.next()
            if batch is None:
                assert other is None
                break
            torch.testing.assert_close(batch["ids"], other["ids"])
            assert batch["reset"] == (batch["position"] == 0)
            assert batch["position"] + batch["ids"].numel() <= 7
            seen.extend(batch["ids"].flatten().tolist())
        assert reader.state_dict() == resumed.state_dict()
    assert sorted(seen) == list(range(37))


def test_batched_epoch_lanes_cover_tokens_and_resume(tmp_path):
    manifest = write_dataset(tmp_path)
    seen = []
    for rank in range(2):
        reader = BatchedEpochTokenStream(manifest, rank, 2, 3, 7, micro_batch_size=2)
        assert reader.rank_chunks[rank] == sum(1 for group in reader.groups
                                               for _ in range(0, int(group[0, 2] - group[0, 1]), 3))
        first = reader.next()
        if first:
            seen.extend(first["ids"].flatten().tolist())
        resumed = BatchedEpochTokenStream(manifest, rank, 2, 3, 7, micro_batch_size=2)
        resumed.load_state_dict(reader.state_dict())
        while True:
            batch, other = reader.next(), resumed.next()
            assert (batch is None) == (other is None)
            if batch is None:
                break
            torch.testing.assert_close(batch["ids"], other["ids"])
            assert batch["position"] == other["position"]
            seen.extend(batch["ids"].flatten().tolist())
        assert reader.state_dict() == resumed.state_dict()
    assert sorted(seen) == list(range(37))
