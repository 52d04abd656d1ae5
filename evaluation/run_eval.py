#!/usr/bin/env python
"""
Run an offline evaluation experiment (models × task sets) and write the results as rows:

    python evaluation/run_eval.py evaluation/experiments/test_config.yaml [--workspace DIR] [--output FILE] [--limit N]

The experiment format and the steps are described in ``olmo_b200/eval/offline.py``.  Results of finished (model, task)
pairs are kept in the workspace folder and reused by later runs.
"""
import argparse
import json
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("experiment")
    ap.add_argument("--workspace", default=None, help="folder for cached step results (overrides the experiment's)")
    ap.add_argument("--output", default=None, help="rows file (.jsonl; a .tsv is written beside it)")
    ap.add_argument("--limit", type=int, default=None, help="cap the documents of every task (smoke runs)")
    ap.add_argument("--device", default=None)
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(name)s %(levelname)s %(message)s")

    from olmo_b200.eval.offline import load_experiment, run_experiment

    spec = load_experiment(args.experiment)
    if args.workspace:
        spec["workspace"] = args.workspace
    if args.output:
        spec["output"] = args.output
    for model in spec["models"]:
        if args.device:
            model["device"] = args.device
        if args.limit is not None:
            model.setdefault("prediction_kwargs", {})["limit"] = args.limit
    rows = run_experiment(spec)
    for row in rows:
        print(json.dumps(row))
    return 0


if __name__ == "__main__":
    sys.exit(main())
