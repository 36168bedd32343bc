#!/usr/bin/env python3
"""Train every full-attention block's TimeMix student in parallel (one teacher pass per step).

Usage: torchrun --standalone --nproc_per_node=N train.py --config configs/train.json [--resume DIR] [--stop-after K]
"""
import argparse
import os

os.environ.setdefault("PYTORCH_ALLOC_CONF", "expandable_segments:True")

from rwkv_theseus_b200.config import load_config  # noqa: E402
from rwkv_theseus_b200.trainer import run  # noqa: E402

if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--config", required=True)
    parser.add_argument("--resume", help="Committed checkpoint directory, output directory, or latest file")
    parser.add_argument("--stop-after", type=int, help="Save and stop after this many optimizer updates")
    args = parser.parse_args()
    run(load_config(args.config), args.resume, args.stop_after)
