#!/usr/bin/env python
"""Move W&B runs whose name matches a regex into another group (reference: ``scripts/wandb_change_group.py``).

    python scripts/wandb_change_group.py ENTITY/PROJECT NAME_REGEX NEW_GROUP [--dry-run]
"""
import re
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.util import positional_args

if __name__ == "__main__":
    project, pattern, group = positional_args(__doc__, 3)[:3]
    import wandb

    for run in wandb.Api().runs(project):
        if re.search(pattern, run.name):
            print(f"{run.name}: {run.group} -> {group}")
            if "--dry-run" not in sys.argv:
                run.group = group
                run.update()
