#!/usr/bin/env python
"""Write an annealing (stage-2 / micro-anneal) config derived from a named recipe or an existing YAML file: linear decay
of the learning rate from the value the base run had reached down to zero over a token budget, starting from a
checkpoint, with a fresh data order (reference: ``scripts/peteish7_config_maker.py``, ``scripts/microanneal_config_maker.py``
).  The data is a named mix, a glob, or a mix assembled here from sources, as those two scripts do:

    python scripts/anneal_config_maker.py --base OLMo2-7B-stage1 --load-path CKPT --start-lr 6.1499e-05 \\
        --tokens 50e9 --name my-anneal --seed 42 -o out.yaml \\
        [--mix MIX --read-location ROOT | --data-glob '/data/anneal/*.npy' |
         --source s3://bucket/dclm/=0.3 --source s3://bucket/math/ --source /data/flan/=2B --source /data/tiny-gsm/=x2]
    python scripts/anneal_config_maker.py --examine out.yaml            # tokens per source of a config's data.paths

``--source PREFIX[=AMOUNT]``: every ``.npy`` file below the prefix (any storage scheme); ``AMOUNT`` is a fraction (``0.3``), a
token count (``2e9``, ``2B``) or a repetition (``x2``).  Files are taken whole in a seeded random order until the amount is
reached (:mod:`olmo_b200.data.mix_builder`).  With ``--tokens auto`` the budget is what the sources add up to (one pass).
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.config import TrainConfig
from olmo_b200.recipes import RECIPES, recipe_dict
from olmo_b200.utils import structured as S


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--examine", metavar="CONFIG", default=None, help="print the per-source token table of CONFIG's data.paths and exit")
    ap.add_argument("--base", required=False, help=f"recipe name ({', '.join(sorted(RECIPES))}) or path of a YAML config")
    ap.add_argument("--load-path")
    ap.add_argument("--start-lr", type=float, help="learning rate of the base run at the checkpoint")
    ap.add_argument("--tokens", help="annealing budget in tokens, or 'auto' for one pass over the assembled sources")
    ap.add_argument("--name")
    ap.add_argument("--source", action="append", default=[], metavar="PREFIX[=AMOUNT]", help="a data source of the mix (repeatable)")
    ap.add_argument("--bytes-per-token", type=int, default=4)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--mix", default=None)
    ap.add_argument("--read-location", default="/data")
    ap.add_argument("--data-glob", default=None)
    ap.add_argument("-o", "--output")
    args = ap.parse_args(argv)
    from olmo_b200.data import mix_builder

    def show(rows) -> None:
        for row in rows:
            print(f"{mix_builder.human_count(row['tokens']):>9}T  {100 * row['share']:5.1f} %  {row['files']:5d} files  {row['source']}")
        print(f"{mix_builder.human_count(sum(r['tokens'] for r in rows)):>9}T  total")

    if args.examine is not None:
        cfg = TrainConfig.load(args.examine, validate_paths=False)
        rows = mix_builder.examine(list(cfg.data.paths or []), bytes_per_token=args.bytes_per_token)
        show(rows)
        return {"rows": rows}
    missing = [flag for flag, value in (("--base", args.base), ("--load-path", args.load_path), ("--start-lr", args.start_lr),
                                        ("--tokens", args.tokens), ("--name", args.name), ("--output", args.output)) if value is None]
    if missing:
        ap.error("missing " + ", ".join(missing))
    mix_paths = mix_rows = None
    if args.source:
        mix_paths, mix_rows = mix_builder.build_mix(args.source, bytes_per_token=args.bytes_per_token, seed=args.seed)
        show(mix_rows)
    if str(args.tokens).lower() == "auto":
        if mix_rows is None:
            ap.error("--tokens auto needs --source")
        args.tokens = float(sum(r["tokens"] for r in mix_rows))
    else:
        args.tokens = float(args.tokens)

    raw = recipe_dict(args.base) if args.base in RECIPES else S.load_yaml(open(args.base))
    seq = raw["model"]["max_sequence_length"]
    batch = raw["global_train_batch_size"]
    steps = round(args.tokens / (batch * seq))
    raw.update(
        run_name=args.name, seed=args.seed, load_path=args.load_path, restore_dataloader=False, no_pre_train_checkpoint=True,
        max_duration=f"{int(args.tokens)}T", stop_at=steps + 10,
        scheduler={"name": "linear_with_warmup", "t_warmup": 0, "alpha_f": 0.0},
    )
    raw["optimizer"] = {**raw["optimizer"], "learning_rate": args.start_lr}
    if mix_paths is not None:
        raw.setdefault("data", {})["paths"] = mix_paths
    elif args.mix is not None:
        from olmo_b200.data.named_data_mixes import resolve_mix

        raw.setdefault("data", {})["paths"] = resolve_mix(args.mix, args.read_location)
    elif args.data_glob is not None:
        raw.setdefault("data", {})["paths"] = "${path.glob:" + args.data_glob + "}"
    Path(args.output).write_text(f"# annealing run derived from {args.base}\n" + S.dump_yaml(raw))
    TrainConfig.load(args.output, validate_paths=False)  # the result must validate
    return raw


if __name__ == "__main__":
    main()
