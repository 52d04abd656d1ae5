#!/usr/bin/env python
"""Print the group of a W&B run given ``entity/project/run_id`` or its URL (reference: ``scripts/group_name_from_wandb.py``)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
from compare_wandb_configs import parse_run_path

if __name__ == "__main__":
    import wandb

    print(wandb.Api().run(parse_run_path(sys.argv[1])).group)
