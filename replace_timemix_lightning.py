#!/usr/bin/env python3
"""Replace chosen mixer layers of a converted Lightning PTH with trained TimeMix weights.

Reads ``migrated.safetensors`` snapshots (a file, or a directory searched recursively in natural path
order; later files win) and writes a new PTH with updated sidecars (see
rwkv_theseus_b200/convert/lightning.py).
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
from rwkv_theseus_b200.convert.lightning import FORMAT, export_tensor, parse_layers, sidecar  # noqa: E402,F401
from rwkv_theseus_b200.convert.lightning import splice_timemix as replace  # noqa: E402

BASE_FORMAT = OUTPUT_FORMAT = FORMAT


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--base", required=True, type=Path, help="converted hybrid .pth")
    p.add_argument("--weights-dir", "--weights", required=True, type=Path,
                   help="Theseus .safetensors file or a directory of snapshots")
    p.add_argument("--layers", required=True, help="decoder layer indices, e.g. 3 or 3,7,11")
    p.add_argument("--out", required=True, type=Path, help="new .pth output path")
    p.add_argument("--head-size", type=int, choices=(64, 128), default=None,
                   help="optional check; each layer's head size is inferred from r_k")
    p.add_argument("--dtype", choices=("base", "source"), default="base",
                   help="cast TimeMix tensors to the base PTH dtype (default) or keep the snapshot dtype")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--verify", action="store_true", help="re-read and byte-check every output tensor")
    p.add_argument("--overwrite", action="store_true")
    p.add_argument("--no-progress", action="store_true")
    a = p.parse_args(argv)
    try:
        replace(a.base, a.weights_dir, a.out, parse_layers(a.layers), head_size=a.head_size, dtype=a.dtype,
                dry_run=a.dry_run, verify=a.verify, overwrite=a.overwrite, quiet=a.no_progress)
    except (OSError, ValueError, KeyError, RuntimeError) as err:
        print(f"ERROR: {err}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
