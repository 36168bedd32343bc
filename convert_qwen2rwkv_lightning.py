#!/usr/bin/env python3
"""Export a LOCAL dense Qwen3.5-family hybrid checkpoint to a Lightning-style PTH.

Only storage layout and names change (see rwkv_theseus_b200/convert/lightning.py); the GDN -> RWKV7
DPLR interpretation is the runtime's. Full attention is retained. Needs torch, safetensors and tqdm;
no Transformers, CUDA or downloads.
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
from rwkv_theseus_b200.convert.lightning import FORMAT, apply, checkpoint_index, geometry, plan  # noqa: E402,F401
from rwkv_theseus_b200.convert.lightning import convert_hf as convert  # noqa: E402


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--src", type=Path, default=Path("./Qwen3.8-27B"), help="LOCAL HF checkpoint directory")
    p.add_argument("--out", type=Path, help="default: SRC/converted/Qwen3.8-27B-RWKV7-Hybrid.pth")
    p.add_argument("--verify", action="store_true", help="re-read the PTH (mmap) and compare every tensor bitwise")
    p.add_argument("--dry-run", action="store_true", help="validate names/shapes/dtypes from headers only")
    p.add_argument("--overwrite", action="store_true", help="replace existing export files")
    p.add_argument("--no-progress", action="store_true")
    p.add_argument("--threads", type=int, default=4, help="CPU threads for repacking/verification")
    a = p.parse_args(argv)
    if a.threads < 1:
        p.error("--threads must be positive")
    import torch
    torch.set_num_threads(a.threads)
    try:
        convert(a.src, a.out or a.src / "converted" / "Qwen3.8-27B-RWKV7-Hybrid.pth", verify=a.verify,
                dry_run=a.dry_run, overwrite=a.overwrite, quiet=a.no_progress)
    except (OSError, ValueError, KeyError, RuntimeError) as err:
        print(f"ERROR: {err}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
