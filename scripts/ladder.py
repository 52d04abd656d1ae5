#!/usr/bin/env python
"""Scaling-ladder front end (reference: ``scripts/ladder.py:381-440``).

    python scripts/ladder.py size --model 1B
    python scripts/ladder.py nodecounts --model 7B [--gpus-per-node 8]
    python scripts/ladder.py dump --model 300M --data MIX --length 2xC --name myrun [--dump_evaluators] [--dump_data]
    torchrun ... scripts/ladder.py train --model 1B --data MIX --length 2xC --name myrun [--read_location /data] [--wandb]
"""
import argparse
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from olmo_b200.ladder import ladder_config, node_counts, size_for_model
from olmo_b200.util import flatten_dict


def config_from_args(args) -> "TrainConfig":  # noqa: F821
    return ladder_config(
        args.model, args.length, args.name, getattr(args, "data", None), read_location=_read_location(args),
        remote_save_folder=(_write_location(args).rstrip("/") + f"/{args.name}-{args.model.upper()}-{args.length}") if _write_location(args) else None,
        load_path=getattr(args, "load_path", None), wandb=getattr(args, "wandb", False), save_overwrite=getattr(args, "save_overwrite", False),
        eval_on_load=getattr(args, "eval_on_load", False),
    )


def _read_location(args) -> str:
    """``--read_location`` wins; ``--s3`` reads from the bucket named by ``OLMO_S3_DATA_ROOT`` (the reference hard-codes its
    own bucket there); otherwise the local data root."""
    if getattr(args, "read_location", None):
        return args.read_location
    if getattr(args, "s3", False):
        return os.environ.get("OLMO_S3_DATA_ROOT", "s3://ai2-llm")
    return "/data"


def _write_location(args):
    if getattr(args, "write_location", None):
        return args.write_location
    if getattr(args, "s3", False):
        return os.environ.get("OLMO_S3_CHECKPOINT_ROOT", "s3://ai2-llm/checkpoints/OLMo-ladder")
    return None


def nodecounts_cmd(args) -> None:
    for n in node_counts(config_from_args(args), args.gpus_per_node):
        print(n)


def size_cmd(args) -> None:
    total, non_embedding = size_for_model(args.model)
    print(total)
    print(non_embedding)


def dump_cmd(args) -> None:
    cfg = config_from_args(args).asdict()
    if not args.dump_evaluators:
        del cfg["evaluators"]
    if not args.dump_data:
        del cfg["data"]
    for key, value in sorted(flatten_dict(cfg).items()):
        print(f"{key}: {value}")


def fit_cmd(args) -> None:
    """Fit ``a * x**b + c`` to the losses in a CSV (``run,loss`` lines; run names as ``train --name`` builds them)."""
    import csv

    from olmo_b200.ladder import ladder_fit

    with open(args.results) as f:
        results = {row[0].strip(): float(row[1]) for row in csv.reader(f) if len(row) >= 2 and not row[0].startswith("#") and row[0] != "run"}
    fit = ladder_fit(results, by=args.by, hold_out=args.hold_out)
    print(f"loss = {fit['a']:.4g} * {args.by}^{fit['b']:.4f} + {fit['c']:.4f}")
    for row in fit["points"]:
        mark = "  (held out)" if row["held_out"] else ""
        print(f"{row['run']:32s} {row['x']:.3e}  loss {row['loss']:.4f}  predicted {row['predicted']:.4f}{mark}")


def train_cmd(args) -> None:
    from train import init_distributed, main
    from olmo_b200.util import prepare_cli_environment

    cfg = config_from_args(args)
    init_distributed()
    prepare_cli_environment()
    main(cfg)


if __name__ == "__main__":
    parser = argparse.ArgumentParser(os.path.basename(__file__), description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = parser.add_subparsers(required=True)
    quiet = dict(data=None, length="1xC", name="nodecounts", wandb=False, save_overwrite=False, load_path=None, eval_on_load=False,
                 read_location=None, write_location=None)
    p = sub.add_parser("nodecounts")
    p.set_defaults(func=nodecounts_cmd, **quiet)
    p.add_argument("--gpus-per-node", type=int, default=8)
    p.add_argument("--model", required=True)
    p = sub.add_parser("size")
    p.set_defaults(func=size_cmd, **quiet)
    p.add_argument("--model", required=True)
    p = sub.add_parser("fit", help="fit a power law to ladder results")
    p.set_defaults(func=fit_cmd)
    p.add_argument("results", help="CSV file of run,loss lines")
    p.add_argument("--by", choices=["size", "length"], default="size")
    p.add_argument("--hold-out", type=int, default=1, help="how many of the largest runs to predict instead of fit")
    dump = sub.add_parser("dump")
    dump.set_defaults(func=dump_cmd)
    dump.add_argument("--dump_evaluators", action=argparse.BooleanOptionalAction, default=False)
    dump.add_argument("--dump_data", action=argparse.BooleanOptionalAction, default=False)
    train = sub.add_parser("train")
    train.set_defaults(func=train_cmd)
    for p in (dump, train):
        p.add_argument("--model", required=True)
        p.add_argument("--data", default=None, help="name of a data mix (see olmo_b200/data/named_data_mixes.py) or a mix file")
        p.add_argument("--length", default="2xC")
        p.add_argument("--name", required=True)
        p.add_argument("--wandb", action=argparse.BooleanOptionalAction, default=False)
        p.add_argument("--s3", action=argparse.BooleanOptionalAction, default=False, help="read data from and write checkpoints to object storage")
        p.add_argument("--read_location", default=None)
        p.add_argument("--write_location", default=None)
        p.add_argument("--save_overwrite", action="store_true")
        p.add_argument("--load_path", default=None)
        p.add_argument("--eval_on_load", action="store_true")
    args = parser.parse_args()
    args.func(args)
