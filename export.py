#!/usr/bin/env python3
"""Write the self-contained export (format 2) of a completed migration checkpoint.

Usage: python export.py --checkpoint RUN_DIR_OR_CHECKPOINT --output EXPORT_DIR
"""
import argparse

from rwkv_theseus_b200.assembly import export_checkpoint

if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--checkpoint", required=True, help="committed checkpoint, its run directory or 'latest'")
    parser.add_argument("--output", required=True, help="directory of the export")
    args = parser.parse_args()
    print(export_checkpoint(args.checkpoint, args.output))
