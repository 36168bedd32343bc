"""Chat JSONL -> manifest v1 conversion: what the readers consume, which conversations are refused and why,
that a failed or refused conversion leaves nothing behind, and that threading never reorders the corpus."""
import json
import threading
import time

import numpy as np
import pytest

from jsonl_to_manifest import convert, validate_messages
from rwkv_theseus_b200.data import EpochTokenStream, sha256_of_file


class LengthTokenizer:
    """ids: the message count, then one id per character of every content field, then an end marker."""

    def __len__(self):
        return 300

    def apply_chat_template(self, messages, tokenize, add_generation_prompt, return_dict):
        assert tokenize and not add_generation_prompt and not return_dict
        ids = [len(messages)]
        for message in messages:
            ids.extend(ord(ch) % 200 for ch in message.get("content", ""))
        return ids + [299]


class ReorderingTokenizer:
    """Lines whose payload is even finish late, so workers complete out of input order."""

    def __init__(self):
        self.threads = set()

    def __len__(self):
        return 300

    def apply_chat_template(self, messages, **_):
        self.threads.add(threading.get_ident())
        payload = int(messages[1]["content"])
        time.sleep(0.003 if payload % 2 == 0 else 0.0)
        return [payload, payload + 100]


def chat(*turns, system=None):
    messages = [{"role": "system", "content": system}] if system else []
    messages += [{"role": role, "content": text} for role, text in turns]
    return {"messages": messages}


def write_jsonl(path, records):
    with path.open("w", encoding="utf-8") as sink:
        for record in records:
            sink.write(json.dumps(record, ensure_ascii=False) + "\n")
    return path


def test_corpus_offsets_and_manifest_fields(tmp_path):
    model = tmp_path / "model"
    model.mkdir()
    (model / "tokenizer_config.json").write_text('{"x": 1}')
    thinking = chat(("user", "hi"), system="sys")
    thinking["messages"].append({"role": "assistant", "reasoning_content": "why", "content": "ok"})
    records = [chat(("user", "ab"), ("assistant", "c")), thinking,
               chat(("user", "q"), ("assistant", "x"), ("tool", "t"), ("assistant", "y"))]
    manifest = convert(write_jsonl(tmp_path / "mix.jsonl", records), model, tmp_path / "built",
                       tokenizer=LengthTokenizer(), progress_interval=0)
    spec = json.loads(manifest.read_text())
    expected = [LengthTokenizer().apply_chat_template(r["messages"], True, False, False) for r in records]
    lengths = [len(ids) for ids in expected]
    source = spec["sources"][0]
    assert spec["format"] == 1 and spec["vocab_size"] == 300
    assert source["name"] == "mix" and source["documents"] == 3 and source["token_count"] == sum(lengths)
    assert spec["tokenizer_files"] == {"tokenizer_config.json": sha256_of_file(model / "tokenizer_config.json")}
    assert source["tokens_sha256"] == sha256_of_file(manifest.parent / source["tokens"])
    np.testing.assert_array_equal(np.load(manifest.parent / source["offsets"]), np.cumsum([0] + lengths))
    np.testing.assert_array_equal(np.fromfile(manifest.parent / source["tokens"], dtype="<u4"),
                                  np.concatenate(expected))
    reader = EpochTokenStream(manifest, 0, 1, chunk_tokens=4, context_tokens=64)
    read = []
    while (batch := reader.next()) is not None:
        read.extend(batch["ids"][0].tolist())
    assert sorted(read) == sorted(np.concatenate(expected).tolist())


@pytest.mark.parametrize("messages, problem", [
    ([], "non-empty array"),
    ([{"role": "assistant", "content": "a"}], "start with a user"),
    ([{"role": "system", "content": "s"}], "contain user and assistant"),
    ([{"role": "user", "content": "u"}, {"role": "assistant", "content": "a", "name": "x"}], "unsupported fields"),
    ([{"role": "user", "content": ""}, {"role": "assistant", "content": "a"}], "non-empty string"),
    ([{"role": "user", "content": "u"}, {"role": "tool", "content": "t"}], "user must be followed by assistant"),
    ([{"role": "user", "content": "u"}, {"role": "assistant", "content": "a"}, {"role": "user", "content": "v"}],
     "must end with assistant"),
    ([{"role": "user", "content": "u"}, {"role": "assistant", "content": "a"}, {"role": "system", "content": "s"}],
     "only allowed as the first"),
    ([{"role": "moderator", "content": "m"}], "role must be one of"),
])
def test_rejected_conversations_name_the_line_and_the_problem(messages, problem):
    with pytest.raises(ValueError, match=problem) as raised:
        validate_messages({"messages": messages}, 12)
    assert "line 12" in str(raised.value)


def test_accepted_shapes():
    validate_messages(chat(("user", "u"), ("assistant", "a")), 1)
    validate_messages(chat(("user", "u"), ("assistant", "a"), ("user", "v"), ("assistant", "b"), system="s"), 2)
    validate_messages(chat(("user", "u"), ("assistant", "a"), ("tool", "t1"), ("tool", "t2"), ("assistant", "b")), 3)


def test_bad_line_or_existing_output_leaves_nothing_new(tmp_path):
    records = [chat(("user", "u"), ("assistant", "a"))] * 3 + [{"messages": "not a list"}]
    source = write_jsonl(tmp_path / "broken.jsonl", records)
    with pytest.raises(ValueError, match="line 4"):
        convert(source, tmp_path, tmp_path / "out", tokenizer=LengthTokenizer(), progress_interval=0)
    assert sorted(p.name for p in tmp_path.iterdir()) == ["broken.jsonl"]
    good = write_jsonl(tmp_path / "good.jsonl", records[:1])
    (tmp_path / "taken").mkdir()
    with pytest.raises(FileExistsError):
        convert(good, tmp_path, tmp_path / "taken", tokenizer=LengthTokenizer(), progress_interval=0)
    assert not any((tmp_path / "taken").iterdir())


def test_worker_count_never_changes_the_corpus(tmp_path):
    source = write_jsonl(tmp_path / "n.jsonl", [chat(("user", "q"), ("assistant", str(i))) for i in range(30)])
    serial = convert(source, tmp_path, tmp_path / "w1", tokenizer=ReorderingTokenizer(), workers=1,
                     progress_interval=0)
    pool_tokenizer = ReorderingTokenizer()
    pooled = convert(source, tmp_path, tmp_path / "w6", tokenizer=pool_tokenizer, workers=6, progress_interval=0)
    assert len(pool_tokenizer.threads) > 1
    assert (serial.parent / "corpus.bin").read_bytes() == (pooled.parent / "corpus.bin").read_bytes()
    ids = np.fromfile(pooled.parent / "corpus.bin", dtype="<u4").reshape(30, 2)
    np.testing.assert_array_equal(ids[:, 0], np.arange(30))
