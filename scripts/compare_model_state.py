#!/usr/bin/env python
"""Diff two checkpoints: parameters (and optionally optimizer moments) that exist on one side only, differ in shape, or
differ in value, largest relative difference first (reference: ``scripts/compare_model_state.py``).

    python scripts/compare_model_state.py BASE_DIR COMPARE_DIR [--optim] [--top 20] [--rtol 0]
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch

from olmo_b200.checkpoint import load_state_dict


def flatten(prefix, obj, out):
    if isinstance(obj, torch.Tensor):
        out[prefix] = obj
    elif isinstance(obj, dict):
        for k, v in obj.items():
            flatten(f"{prefix}.{k}" if prefix else str(k), v, out)
    return out


def compare(a: dict, b: dict, top: int, rtol: float) -> int:
    only_a, only_b = sorted(set(a) - set(b)), sorted(set(b) - set(a))
    for name in only_a:
        print(f"only in base:    {name}")
    for name in only_b:
        print(f"only in compare: {name}")
    rows = []
    for name in sorted(set(a) & set(b)):
        x, y = a[name], b[name]
        if x.shape != y.shape:
            print(f"shape differs:   {name}: {tuple(x.shape)} vs {tuple(y.shape)}")
            continue
        x, y = x.float(), y.float()
        diff = (x - y).norm().item()
        rel = diff / max(x.norm().item(), 1e-12)
        if rel > rtol:
            rows.append((rel, diff, (x - y).abs().max().item(), name))
    rows.sort(reverse=True)
    for rel, diff, mx, name in rows[:top]:
        print(f"{name}: rel {rel:.3e}  l2 {diff:.3e}  max {mx:.3e}")
    print(f"{len(rows)} of {len(set(a) & set(b))} shared tensors differ (rtol {rtol})")
    return len(rows) + len(only_a) + len(only_b)


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("base")
    ap.add_argument("compare")
    ap.add_argument("--optim", action="store_true", help="also compare optim.pt")
    ap.add_argument("--top", type=int, default=20)
    ap.add_argument("--rtol", type=float, default=0.0)
    args = ap.parse_args()
    bad = compare(flatten("", load_state_dict(args.base, "model.pt", map_location="cpu"), {}),
                  flatten("", load_state_dict(args.compare, "model.pt", map_location="cpu"), {}), args.top, args.rtol)
    if args.optim:
        bad += compare(flatten("", load_state_dict(args.base, "optim.pt", map_location="cpu"), {}),
                       flatten("", load_state_dict(args.compare, "optim.pt", map_location="cpu"), {}), args.top, args.rtol)
    sys.exit(1 if bad else 0)
