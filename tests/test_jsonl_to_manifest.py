"""Chat JSONL -> manifest v1 tool: reader-compatible output, explicit schema errors, atomic output,
order-preserving threaded tokenisation (the reference's ``tests/test_jsonl_to_manifest.py`` contract)."""
import json
import random
import time

import numpy as np
import pytest

from jsonl_to_manifest import convert, validate_messages
from rwkv_theseus_b200.data import TokenStream


class CountingTokenizer:
    """Emits three ids that depend on the number of messages."""

    def __len__(self):
        return 256

    def apply_chat_template(self, messages, **kwargs):
        assert kwargs == {"tokenize": True, "add_generation_prompt": False, "return_dict": False}
        n = len(messages)
        return [10 + n, 20 + n, 2]


class SlowJitterTokenizer:
    """Finishes lines out of order (random sleeps); ids encode the line's payload."""

    def __len__(self):
        return 256

    def apply_chat_template(self, messages, **kwargs):
        value = int(messages[-1]["content"])
        time.sleep(random.Random(value).random() * 0.004)
        return [value, 255 - value]


def conversation(*pairs, system=None):
    msgs = [{"role": "system", "content": system}] if system else []
    for role, content in pairs:
        msgs.append({"role": role, "content": content})
    return {"messages": msgs}


def write(path, rows):
    path.write_text("".join(json.dumps(r, ensure_ascii=False) + "\n" for r in rows), encoding="utf-8")


def test_output_is_a_reader_compatible_manifest(tmp_path):
    tok = tmp_path / "model"
    tok.mkdir()
    (tok / "tokenizer.json").write_text("{}")
    src = tmp_path / "train.jsonl"
    reasoning = conversation(("user", "u"), system="s")
    reasoning["messages"].append({"role": "assistant", "reasoning_content": "r", "content": "a"})
    write(src, [conversation(("user", "u"), ("assistant", "a")), reasoning])
    manifest_path = convert(src, tok, tmp_path / "out", tokenizer=CountingTokenizer(), progress_interval=0)
    manifest = json.loads(manifest_path.read_text())
    source = manifest["sources"][0]
    assert manifest["format"] == 1 and manifest["vocab_size"] == 256
    assert (source["documents"], source["token_count"], source["name"]) == (2, 6, "train")
    assert len(manifest["tokenizer_files"]["tokenizer.json"]) == 64
    np.testing.assert_array_equal(np.load(tmp_path / "out" / "corpus.offsets.npy"), [0, 3, 6])
    np.testing.assert_array_equal(np.fromfile(tmp_path / "out" / "corpus.bin", dtype="<u4"), [12, 22, 2, 13, 23, 2])
    stream = TokenStream(manifest_path, pair_id=0, pairs=1, chunk_tokens=8, context_tokens=8)
    assert stream.next()["ids"].shape == (1, 3)


@pytest.mark.parametrize("messages, text", [
    ([{"role": "assistant", "content": "a"}], "start with a user"),
    ([{"role": "user", "content": "u"}], "contain user and assistant"),
    ([{"role": "user", "content": "u"}, {"role": "assistant", "content": "a", "extra": 1}], "unsupported fields"),
    ([{"role": "user", "content": "u"}, {"role": "assistant", "content": " "}], "non-empty string"),
    ([{"role": "user", "content": "u"}, {"role": "user", "content": "v"}], "user must be followed by assistant"),
    ([{"role": "user", "content": "u"}, {"role": "assistant", "content": "a"}, {"role": "tool", "content": "t"}],
     "must end with assistant"),
    ([{"role": "user", "content": "u"}, {"role": "system", "content": "s"}], "only allowed as the first"),
    ([{"role": "robot", "content": "u"}], "role must be one of"),
])
def test_schema_errors_name_the_problem(messages, text):
    with pytest.raises(ValueError, match=text):
        validate_messages({"messages": messages}, 7)
    with pytest.raises(ValueError, match="line 7"):
        validate_messages({"messages": messages}, 7)


def test_tool_turns_are_accepted():
    validate_messages(conversation(("user", "u"), ("assistant", "a"), ("tool", "t"), ("tool", "t2"),
                                   ("assistant", "b")), 1)


def test_failed_conversion_leaves_no_output(tmp_path):
    src = tmp_path / "bad.jsonl"
    src.write_text("{}\n", encoding="utf-8")
    with pytest.raises(ValueError, match="line 1"):
        convert(src, tmp_path, tmp_path / "out", tokenizer=CountingTokenizer(), progress_interval=0)
    assert not (tmp_path / "out").exists() and not (tmp_path / "out.building").exists()


def test_existing_output_is_refused(tmp_path):
    src = tmp_path / "a.jsonl"
    write(src, [conversation(("user", "u"), ("assistant", "a"))])
    (tmp_path / "out").mkdir()
    with pytest.raises(FileExistsError):
        convert(src, tmp_path, tmp_path / "out", tokenizer=CountingTokenizer(), progress_interval=0)


def test_threaded_output_is_byte_identical_and_ordered(tmp_path):
    src = tmp_path / "train.jsonl"
    write(src, [conversation(("user", "u"), ("assistant", str(i))) for i in range(24)])
    one = convert(src, tmp_path, tmp_path / "one", tokenizer=SlowJitterTokenizer(), workers=1, progress_interval=0)
    many = convert(src, tmp_path, tmp_path / "many", tokenizer=SlowJitterTokenizer(), workers=8,
                   progress_interval=0)
    assert (one.parent / "corpus.bin").read_bytes() == (many.parent / "corpus.bin").read_bytes()
    tokens = np.fromfile(many.parent / "corpus.bin", dtype="<u4").reshape(-1, 2)
    np.testing.assert_array_equal(tokens[:, 0], np.arange(24))
