#!/usr/bin/env python
"""Move W&B runs whose name matches a regex into another group (reference: ``scripts/wandb_change_group.py``).

    python scripts/wandb_change_group.py ENTITY/PROJECT NAME_REGEX NEW_GROUP [--dry-run]
"""
import re
import sys

if __name__ == "__main__":
    if len(sys.argv) < 4:
        raise SystemExit(__doc__)
    import wandb

    project, pattern, group = sys.argv[1:4]
    for run in wandb.Api().runs(project):
        if re.search(pattern, run.name):
            print(f"{run.name}: {run.group} -> {group}")
            if "--dry-run" not in sys.argv:
                run.group = group
                run.update()
