#!/usr/bin/env python3
"""Validate a committed checkpoint on every launched rank (metrics summed over ranks).

Usage: torchrun --standalone --nproc_per_node=N validate.py --config configs/train.json --checkpoint RUN_DIR
"""
import argparse

from rwkv_theseus_b200.assembly import validate_checkpoint
from rwkv_theseus_b200.config import load_config

if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--config", required=True)
    parser.add_argument("--checkpoint", required=True, help="committed checkpoint, its run directory or 'latest'")
    args = parser.parse_args()
    validate_checkpoint(load_config(args.config), args.checkpoint)
