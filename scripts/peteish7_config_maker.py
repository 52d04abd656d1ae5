#!/usr/bin/env python
"""Mid-training (50B / 100B / 300B token) anneal configs for the 7B run, assembled from data sources.

The name of the reference's tool for this; the work is done by ``scripts/anneal_config_maker.py`` with the 7B stage-1 recipe
as the base and its endpoint as the default starting point.

    python scripts/peteish7_config_maker.py --name my-anneal --tokens 50e9 -o configs/annealing/my-anneal.yaml \\
        --source s3://bucket/dclm/=0.47 --source s3://bucket/flan/=0.17 --source s3://bucket/math/ [--start-lr LR] [--load-path CKPT]
    python scripts/peteish7_config_maker.py --examine configs/annealing/my-anneal.yaml
"""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from anneal_config_maker import main as make

DEFAULTS = {"--base": "OLMo2-7B-stage1", "--start-lr": "6.1499e-05", "--seed": "42",
            "--load-path": "${oc.env:OLMO_STAGE1_CHECKPOINT,https://olmo-checkpoints.org/ai2-llm/peteish7/step928646-unsharded}"}


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--examine" not in argv:
        for flag, value in DEFAULTS.items():
            if flag not in argv:
                argv += [flag, value]
    return make(argv)


if __name__ == "__main__":
    main()
