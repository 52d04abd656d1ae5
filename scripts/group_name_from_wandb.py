#!/usr/bin/env python
"""Print the group of a W&B run given ``entity/project/run_id`` or its URL (reference: ``scripts/group_name_from_wandb.py``)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(1, str(Path(__file__).resolve().parent.parent))
from compare_wandb_configs import parse_run_path

from olmo_b200.util import positional_args

if __name__ == "__main__":
    (run_path,) = positional_args(__doc__, 1)[:1]
    import wandb

    print(wandb.Api().run(parse_run_path(run_path)).group)
