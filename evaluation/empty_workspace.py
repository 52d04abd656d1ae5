#!/usr/bin/env python
"""Forget cached evaluation steps: ``python evaluation/empty_workspace.py WORKSPACE [--yes]`` removes the per-(model, task)
result files of a workspace folder so that the next run recomputes them (the reference's script of this name empties a
workflow-engine workspace)."""
import argparse
import sys
from pathlib import Path


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("workspace")
    ap.add_argument("--yes", action="store_true", help="do not ask")
    args = ap.parse_args(argv)
    files = sorted(Path(args.workspace).glob("*.json")) if Path(args.workspace).is_dir() else []
    if not files:
        print("nothing to remove")
        return 0
    if not args.yes and input(f"remove {len(files)} cached results from {args.workspace}? [y/N] ").strip().lower() not in ("y", "yes"):
        print("cancelled")
        return 1
    for f in files:
        f.unlink()
    print(f"removed {len(files)} cached results")
    return 0


if __name__ == "__main__":
    sys.exit(main())
