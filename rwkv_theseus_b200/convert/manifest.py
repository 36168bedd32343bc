"""Chat JSONL -> token manifest v1 (reference ``jsonl_to_manifest.py:1-299``).

Input: UTF-8 JSONL, one conversation per line: ``{"messages": [{"role", "content"}, ...]}``
with roles system (first message only), user, assistant (may also carry ``reasoning_content``)
and tool, in the order system? (user assistant (tool* assistant)* )+ ... ending with assistant.
Each conversation is rendered with the tokenizer's chat template
(``apply_chat_template(messages, tokenize=True, add_generation_prompt=False, return_dict=False)``)
and appended to ``corpus.bin`` (little-endian uint32); ``corpus.offsets.npy`` (int64) holds the
document boundaries. The output directory is built as ``<out>.building`` and renamed into place
only when complete; any failure removes it.

Tokenisation runs on a thread pool with a bounded window of in-flight lines; results are
written strictly in input order, so the corpus is byte-identical for any worker count.
"""
import collections
import hashlib
import json
import math
import os
import shutil
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

TOKENIZER_FILES = frozenset({"added_tokens.json", "chat_template.jinja", "merges.txt", "special_tokens_map.json",
                             "tokenizer.json", "tokenizer.model", "tokenizer_config.json", "vocab.json"})
# role -> roles allowed to follow it; None stands for "conversation start (or after the system prompt)"
_NEXT = {None: {"user"}, "system": {"user"}, "user": {"assistant"}, "assistant": {"user", "tool"},
         "tool": {"tool", "assistant"}}
_FIELDS = {"system": {"role", "content"}, "user": {"role", "content"}, "tool": {"role", "content"},
           "assistant": {"role", "content", "reasoning_content"}}
_CHUNK = 8 << 20


def file_sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while block := f.read(_CHUNK):
            h.update(block)
    return h.hexdigest()


def validate_messages(record, line_number):
    """Return the conversation's messages after checking the fixed schema; ValueError names the line."""
    where = f"line {line_number}"
    if not isinstance(record, dict):
        raise ValueError(f"{where}: top-level JSON value must be an object")
    messages = record.get("messages")
    if not isinstance(messages, list) or not messages:
        raise ValueError(f"{where}: 'messages' must be a non-empty array")
    previous = None
    for i, message in enumerate(messages):
        at = f"{where}, messages[{i}]"
        if not isinstance(message, dict):
            raise ValueError(f"{at}: message must be an object")
        role = message.get("role")
        if role not in _FIELDS:
            raise ValueError(f"{at}: role must be one of {sorted(_FIELDS)}")
        extra = set(message) - _FIELDS[role]
        if extra:
            raise ValueError(f"{at}: unsupported fields: {sorted(extra)}")
        content = message.get("content")
        if not isinstance(content, str) or not content.strip():
            raise ValueError(f"{at}: content must be a non-empty string")
        if "reasoning_content" in message and not isinstance(message["reasoning_content"], str):
            raise ValueError(f"{at}: reasoning_content must be a string")
        if role == "system":
            if i:
                raise ValueError(f"{at}: system is only allowed as the first message")
        elif role not in _NEXT[previous]:
            if previous in (None, "system"):
                raise ValueError(f"{at}: the conversation must start with a user message")
            raise ValueError(f"{at}: {previous} must be followed by {' or '.join(sorted(_NEXT[previous]))}")
        previous = role
    roles = {m["role"] for m in messages}
    if not {"user", "assistant"} <= roles:
        raise ValueError(f"{where}: conversation must contain user and assistant messages")
    if previous != "assistant":
        raise ValueError(f"{where}: a complete training conversation must end with assistant")
    return messages


def tokenize_line(line_number, line, tokenizer, vocab_size):
    if not line.strip():
        raise ValueError(f"line {line_number}: blank lines are not allowed")
    try:
        record = json.loads(line)
    except json.JSONDecodeError as err:
        raise ValueError(f"line {line_number}: invalid JSON: {err.msg}") from err
    messages = validate_messages(record, line_number)
    try:
        ids = tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=False, return_dict=False)
    except Exception as err:  # the tokenizer's own failure, reported with the line
        raise ValueError(f"line {line_number}: chat template/tokenization failed: {err}") from err
    ids = ids.tolist() if hasattr(ids, "tolist") else ids
    if not isinstance(ids, list) or not ids:
        raise ValueError(f"line {line_number}: tokenizer returned an empty or invalid token list")
    if not all(isinstance(t, (int, np.integer)) and not isinstance(t, bool) for t in ids):
        raise ValueError(f"line {line_number}: tokenizer returned a non-integer token ID")
    arr = np.asarray(ids, dtype=np.int64)
    if arr.min() < 0 or arr.max() >= vocab_size:
        raise ValueError(f"line {line_number}: token ID is outside tokenizer vocabulary [0, {vocab_size})")
    return arr.astype("<u4")


def tokenize_in_order(lines, tokenizer, vocab_size, workers):
    """Yield token arrays in input order; at most 2 * workers lines are in flight."""
    numbered = enumerate(lines, 1)
    if workers == 1:
        for number, line in numbered:
            yield tokenize_line(number, line, tokenizer, vocab_size)
        return
    window = collections.deque()
    with ThreadPoolExecutor(workers, thread_name_prefix="tokenize") as pool:
        try:
            for number, line in numbered:
                window.append(pool.submit(tokenize_line, number, line, tokenizer, vocab_size))
                if len(window) >= 2 * workers:
                    yield window.popleft().result()
            while window:
                yield window.popleft().result()
        finally:
            for future in window:
                future.cancel()


def _scan(path):
    """(sha256, line count, (size, mtime_ns)) of the input, read once before converting."""
    h, newlines, last = hashlib.sha256(), 0, b""
    with open(path, "rb") as f:
        while block := f.read(_CHUNK):
            h.update(block)
            newlines += block.count(b"\n")
            last = block[-1:]
    st = path.stat()
    return h.hexdigest(), newlines + (st.st_size > 0 and last != b"\n"), (st.st_size, st.st_mtime_ns)


def tokenizer_hashes(directory):
    directory = Path(directory)
    if not directory.is_dir():
        return {}
    return {p.relative_to(directory).as_posix(): file_sha256(p)
            for p in sorted(directory.rglob("*")) if p.is_file() and p.name in TOKENIZER_FILES}


def convert(input_path, tokenizer_path, output_path, *, weight=1.0, name=None, progress_interval=1, workers=None,
            tokenizer=None):
    """Build ``output_path`` (a new directory) and return the path of its manifest.json."""
    src, tok_dir, out = (Path(p).resolve() for p in (input_path, tokenizer_path, output_path))
    building = out.with_name(out.name + ".building")
    if not src.is_file():
        raise FileNotFoundError(f"input JSONL does not exist: {src}")
    if not tok_dir.is_dir():
        raise FileNotFoundError(f"local tokenizer directory does not exist: {tok_dir}")
    for path, what in ((out, "output"), (building, "temporary output")):
        if path.exists():
            raise FileExistsError(f"{what} already exists: {path}")
    weight = float(weight)
    workers = int(os.cpu_count() or 1) if workers is None else int(workers)
    problems = [text for bad, text in ((not math.isfinite(weight) or weight <= 0, f"source weight {weight} is not a "
                                        "positive finite number"),
                                       (workers < 1, f"need at least one tokenizer worker, got {workers}"),
                                       (progress_interval < 0, f"negative progress_interval {progress_interval}"))
                if bad]
    if problems:
        raise ValueError("; ".join(problems))
    if tokenizer is None:
        from transformers import AutoTokenizer
        tokenizer = AutoTokenizer.from_pretrained(tok_dir, local_files_only=True)
    vocab_size = int(len(tokenizer))
    if not 0 < vocab_size <= np.iinfo(np.uint32).max:
        raise ValueError(f"tokenizer size cannot be represented as uint32: {vocab_size}")
    input_sha, total_lines, stamp = _scan(src)
    out.parent.mkdir(parents=True, exist_ok=True)
    building.mkdir()
    try:
        from tqdm.auto import tqdm
        tokens_path, offsets_path = building / "corpus.bin", building / "corpus.offsets.npy"
        offsets = [0]
        with open(src, encoding="utf-8") as lines, open(tokens_path, "wb") as sink, \
                tqdm(total=total_lines, desc=f"tokenize ({workers} threads)", unit="doc",
                     miniters=max(1, progress_interval), disable=progress_interval == 0) as bar:
            for arr in tokenize_in_order(lines, tokenizer, vocab_size, workers):
                sink.write(arr.tobytes())
                offsets.append(offsets[-1] + len(arr))
                bar.update(1)
        documents = len(offsets) - 1
        if documents == 0:
            raise ValueError("input JSONL contains no documents")
        st = src.stat()
        if (st.st_size, st.st_mtime_ns) != stamp:
            raise RuntimeError("input JSONL changed during conversion")
        np.save(offsets_path, np.asarray(offsets, dtype=np.int64), allow_pickle=False)
        manifest = {"format": 1, "vocab_size": vocab_size, "tokenizer": str(tok_dir),
                    "tokenizer_files": tokenizer_hashes(tok_dir),
                    "sources": [{"name": name or src.stem, "tokens": tokens_path.name, "offsets": offsets_path.name,
                                 "weight": weight, "documents": documents, "token_count": offsets[-1],
                                 "input_sha256": input_sha, "tokens_sha256": file_sha256(tokens_path),
                                 "offsets_sha256": file_sha256(offsets_path)}]}
        (building / "manifest.json").write_text(json.dumps(manifest, ensure_ascii=False, indent=2) + "\n",
                                                encoding="utf-8")
        os.replace(building, out)
    except BaseException:
        shutil.rmtree(building, ignore_errors=True)
        raise
    print(f"wrote {documents:,} documents / {offsets[-1]:,} tokens to {out}")
    return out / "manifest.json"
