#!/usr/bin/env python
"""List the rendered-request evaluation dumps found in the packaged-data tree (``oe_eval_tasks/<task>/<variant>/``) with
their request counts and primary metrics, and say which of them have a label in the task table (reference:
``scripts/list_evals_from_oe_eval.py`` printed the table entries to paste; here the table is generated, so this is a check)."""
import gzip
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.eval.downstream import METRIC_FROM_OE_EVAL, label_to_task_map
from olmo_b200.util import get_data_path

def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--num-examples", type=int, default=0, help="also print this many rendered requests of every dump")
    args = ap.parse_args(argv)
    try:
        root = get_data_path("oe_eval_tasks")
    except FileNotFoundError as e:
        raise SystemExit(str(e))
    shown = 0
    for cfg_file in sorted(list(root.glob("*/*/config.json")) + list(root.glob("*/config.json"))):
        nested = cfg_file.parent.parent != root
        task, variant = (cfg_file.parent.parent.name, cfg_file.parent.name) if nested else (cfg_file.parent.name, None)
        cfg = json.loads(cfg_file.read_text())
        metric = METRIC_FROM_OE_EVAL.get(cfg.get("task_config", {}).get("primary_metric"), "?")
        n, examples = 0, []
        for req in sorted(cfg_file.parent.glob("*requests.jsonl.gz")):
            with gzip.open(req, "rt") as f:
                for line in f:
                    if len(examples) < args.num_examples:
                        examples.append(json.loads(line))
                    n += 1
        label = f"{task}_{variant}" if variant else task
        print(f"{label:45s} metric={metric:9s} requests={n:7d} {'in table' if label in label_to_task_map else 'NOT in table'}")
        for i, example in enumerate(examples):
            print(f"  example {i}: {example}")
        shown += 1
    return shown


if __name__ == "__main__":
    main()
