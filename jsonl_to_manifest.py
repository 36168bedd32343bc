#!/usr/bin/env python3
"""Convert fixed-schema conversation JSONL to a token manifest v1 (see rwkv_theseus_b200/convert/manifest.py)."""
import argparse
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
from rwkv_theseus_b200.convert.manifest import convert, tokenize_in_order, validate_messages  # noqa: E402,F401


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--input", required=True, help="UTF-8 JSONL input file")
    p.add_argument("--tokenizer", required=True, help="local HF model/tokenizer directory")
    p.add_argument("--output", required=True, help="new output directory (must not exist)")
    p.add_argument("--name", help="source name stored in the manifest")
    p.add_argument("--weight", type=float, default=1.0, help="source sampling weight")
    p.add_argument("--workers", type=int, default=os.cpu_count() or 1, help="tokenisation threads")
    p.add_argument("--progress-interval", type=int, default=1, help="documents per progress update; 0 disables it")
    a = p.parse_args(argv)
    if a.workers < 1:
        p.error("--workers must be >= 1")
    if a.progress_interval < 0:
        p.error("--progress-interval must be >= 0")
    convert(a.input, a.tokenizer, a.output, weight=a.weight, name=a.name, progress_interval=a.progress_interval,
            workers=a.workers)


if __name__ == "__main__":
    main()
