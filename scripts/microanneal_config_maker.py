#!/usr/bin/env python
"""Micro-anneal configs (one pass over a small candidate source mixed with web text, to rank data sources cheaply).

The name of the reference's tool for this; the work is done by ``scripts/anneal_config_maker.py`` with the settings those runs
share: the 7B stage-1 endpoint as starting point unless ``--load-path`` says otherwise, its learning rate there (6.1499e-05)
unless ``--start-lr`` is given, a budget of one pass over the assembled sources.

    python scripts/microanneal_config_maker.py --name my-source -o configs/microannealing/my-source.yaml \\
        --source s3://bucket/candidate/ --source s3://bucket/dclm/=0.01 [--load-path CKPT] [--start-lr LR] [--seed 7201]
    python scripts/microanneal_config_maker.py --examine configs/microannealing/my-source.yaml
"""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from anneal_config_maker import main as make

DEFAULTS = {"--base": "OLMo2-7B-stage1", "--start-lr": "6.1499e-05", "--tokens": "auto", "--seed": "7201",
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
