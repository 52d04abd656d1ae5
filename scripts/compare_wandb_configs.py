#!/usr/bin/env python
"""Print the config keys on which two W&B runs differ (``entity/project/run_id`` or run URLs), skipping keys that always
differ such as save folders and timestamps (reference: ``scripts/compare_wandb_configs.py``)."""
import re
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.util import flatten_dict, positional_args

NOISE = re.compile(r"(save_folder|remote_save_folder|load_path|run_name|wandb\.|time_limit|_wandb)")


def parse_run_path(s: str) -> str:
    m = re.match(r"^(?:https?://wandb\.ai/)?([^/]+)/([^/]+)/(?:runs/)?([^/?]+)", s.strip())
    if m is None:
        raise ValueError(f"cannot parse W&B run '{s}'")
    return "/".join(m.groups())


def diff(a: dict, b: dict, show_noise: bool = False):
    fa, fb = flatten_dict(a, include_lists=True), flatten_dict(b, include_lists=True)
    for key in sorted(set(fa) | set(fb)):
        if not show_noise and NOISE.search(key):
            continue
        va, vb = fa.get(key, "<missing>"), fb.get(key, "<missing>")
        if va != vb:
            yield key, va, vb


if __name__ == "__main__":
    args = positional_args((__doc__ or "") + "\n\n    python scripts/compare_wandb_configs.py RUN_A RUN_B [--all]", 2)
    import wandb

    api = wandb.Api()
    left, right = (api.run(parse_run_path(s)) for s in args[:2])
    for key, va, vb in diff(left._attrs["rawconfig"], right._attrs["rawconfig"], "--all" in args):
        print(f"{key}\n\t{va}\n\t{vb}")
