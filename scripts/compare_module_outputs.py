#!/usr/bin/env python
"""Diff the per-module input/output dumps that ``module_outputs_save_steps`` writes under ``traces/step{N}/`` for two runs
and report where they first diverge (reference: ``scripts/compare_module_outputs.py``).

    python scripts/compare_module_outputs.py RUN_A/traces/step1 RUN_B/traces/step1 [--rtol 1e-3] [--verbose]
                                             [--include_non_tensor_outputs]

Dumps whose content is not made of tensors (for example an attention layer's cache entry of ``None``) are skipped unless
``--include_non_tensor_outputs``, with which they are compared for equality.
"""
import argparse
import re
import sys
from pathlib import Path

import torch


def order_key(path: Path):
    # files are named "<module path>_{input,output}.pt" (+ "_mb<k>" for micro-batches); blocks sort numerically
    parts = [int(p) if p.isdigit() else p for p in re.split(r"[._]", path.stem)]
    return [(0, p) if isinstance(p, int) else (1, p) for p in parts]


def tensors(obj):
    if isinstance(obj, torch.Tensor):
        yield obj
    elif isinstance(obj, (list, tuple)):
        for x in obj:
            yield from tensors(x)
    elif isinstance(obj, dict):
        for x in obj.values():
            yield from tensors(x)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("base")
    ap.add_argument("compare")
    ap.add_argument("--rtol", type=float, default=1e-3)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--include_non_tensor_outputs", action="store_true", help="also compare dumps that hold no tensors, by equality")
    args = ap.parse_args()
    a_dir, b_dir = Path(args.base), Path(args.compare)
    a_files = {p.name: p for p in a_dir.glob("*.pt")}
    b_files = {p.name: p for p in b_dir.glob("*.pt")}
    for name in sorted(set(a_files) ^ set(b_files)):
        print(f"only in {'base' if name in a_files else 'compare'}: {name}")
    first_bad = None
    for name in sorted(set(a_files) & set(b_files), key=lambda n: order_key(a_files[n])):
        raw_a = torch.load(a_files[name], map_location="cpu", weights_only=False)
        raw_b = torch.load(b_files[name], map_location="cpu", weights_only=False)
        xa, xb = list(tensors(raw_a)), list(tensors(raw_b))
        if not xa and not xb:
            if args.include_non_tensor_outputs:
                same = raw_a == raw_b
                if not same and first_bad is None:
                    first_bad = name
                if not same or args.verbose:
                    print(f"{'ok  ' if same else 'DIFF'} {name}: {raw_a!r} vs {raw_b!r}")
            continue
        worst = 0.0 if len(xa) == len(xb) else float("inf")
        for x, y in zip(xa, xb):
            if x.shape != y.shape:
                worst = float("inf")
                break
            x, y = x.float(), y.float()
            worst = max(worst, ((x - y).norm() / x.norm().clamp_min(1e-12)).item())
        flag = worst > args.rtol
        if flag and first_bad is None:
            first_bad = name
        if flag or args.verbose:
            print(f"{'DIFF' if flag else 'ok  '} {name}: rel {worst:.3e}")
    print(f"first divergence: {first_bad}" if first_bad else "no divergence above tolerance")
    return 1 if first_bad else 0


if __name__ == "__main__":
    sys.exit(main())
