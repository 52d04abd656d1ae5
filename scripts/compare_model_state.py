#!/usr/bin/env python
"""Diff two checkpoints: parameters (and optionally optimizer moments) that exist on one side only, differ in shape, or
differ in value, largest relative difference first (reference: ``scripts/compare_model_state.py``).

    python scripts/compare_model_state.py BASE_DIR COMPARE_DIR [--optim] [--top 20] [--rtol 0] [--norm_order 2]
                                          [--skip_non_tensor_state] [--verbose]

``--norm_order`` picks the vector norm of the reported differences; non-tensor entries of the optimizer state (step counts,
group settings) are compared for equality unless ``--skip_non_tensor_state``; ``--verbose`` also lists dtype changes and the
tensors that agree.
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch

from olmo_b200.checkpoint import load_state_dict


def flatten(prefix, obj, out, others=None):
    """Tensors by dotted path into ``out``; with ``others`` given, every other leaf goes there."""
    if isinstance(obj, torch.Tensor):
        out[prefix] = obj
    elif isinstance(obj, dict):
        for k, v in obj.items():
            flatten(f"{prefix}.{k}" if prefix else str(k), v, out, others)
    elif isinstance(obj, (list, tuple)) and others is not None:
        for i, v in enumerate(obj):
            flatten(f"{prefix}.{i}", v, out, others)
    elif others is not None:
        others[prefix] = obj
    return out


def compare_plain(a: dict, b: dict) -> int:
    """Non-tensor leaves: report what is missing on a side or unequal."""
    bad = 0
    for name in sorted(set(a) | set(b)):
        if name not in a or name not in b:
            print(f"only in {'base' if name in a else 'compare'}: {name}")
            bad += 1
        elif a[name] != b[name]:
            print(f"value differs:   {name}: {a[name]!r} vs {b[name]!r}")
            bad += 1
    return bad


def compare(a: dict, b: dict, top: int, rtol: float, norm_order: float = 2, verbose: bool = False) -> int:
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
        if verbose and x.dtype != y.dtype:
            print(f"dtype differs:   {name}: {x.dtype} vs {y.dtype}")
        x, y = x.float(), y.float()
        diff = torch.linalg.vector_norm(x - y, ord=norm_order).item()
        rel = diff / max(torch.linalg.vector_norm(x, ord=norm_order).item(), 1e-12)
        if rel > rtol:
            rows.append((rel, diff, (x - y).abs().max().item(), name))
        elif verbose:
            print(f"same:            {name}")
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
    ap.add_argument("--norm_order", type=float, default=2, help="order of the vector norm the differences are measured in")
    ap.add_argument("--skip_non_tensor_state", action="store_true", help="do not compare step counts, group settings and other plain values")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    bad = compare(flatten("", load_state_dict(args.base, "model.pt", map_location="cpu"), {}),
                  flatten("", load_state_dict(args.compare, "model.pt", map_location="cpu"), {}), args.top, args.rtol, args.norm_order, args.verbose)
    if args.optim:
        plain_a, plain_b = {}, {}
        bad += compare(flatten("", load_state_dict(args.base, "optim.pt", map_location="cpu"), {}, plain_a),
                       flatten("", load_state_dict(args.compare, "optim.pt", map_location="cpu"), {}, plain_b), args.top, args.rtol,
                       args.norm_order, args.verbose)
        if not args.skip_non_tensor_state:
            bad += compare_plain(plain_a, plain_b)
    sys.exit(1 if bad else 0)
