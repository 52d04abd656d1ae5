#!/usr/bin/env python
"""Print the learning rate a W&B-logged run used at a given step (``optim/learning_rate_group0``), which is what an
annealing run needs as its starting LR (reference: ``scripts/learning_rate_at_step_from_wandb.py``).

    python scripts/learning_rate_at_step_from_wandb.py ENTITY/PROJECT/RUN_ID STEP
"""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(1, str(Path(__file__).resolve().parent.parent))
from compare_wandb_configs import parse_run_path

from olmo_b200.util import positional_args

if __name__ == "__main__":
    run_path, step_text = positional_args(__doc__, 2)[:2]
    import wandb

    run = wandb.Api().run(parse_run_path(run_path))
    step = int(step_text)
    key = "optim/learning_rate_group0"
    rows = run.scan_history(keys=[key, "_step"], min_step=step, max_step=step + 1, page_size=5)
    for row in rows:
        if row["_step"] == step:
            print(row[key])
            break
    else:
        raise SystemExit(f"no {key} logged at step {step}")
