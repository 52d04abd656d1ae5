#!/usr/bin/env python
"""Write an annealing (stage-2 / micro-anneal) config derived from a named recipe or an existing YAML file: linear decay
of the learning rate from the value the base run had reached down to zero over a token budget, starting from a
checkpoint, with a fresh data order (reference: ``scripts/peteish7_config_maker.py``, ``scripts/microanneal_config_maker.py``
— those assemble source mixes for AI2's buckets; here the data mix is a named mix, a mix file, or ``--data-glob``).

    python scripts/anneal_config_maker.py --base OLMo2-7B-stage1 --load-path CKPT --start-lr 6.1499e-05 \\
        --tokens 50e9 --name my-anneal --seed 42 [--mix MIX --read-location ROOT | --data-glob '/data/anneal/*.npy'] -o out.yaml
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
    ap.add_argument("--base", required=True, help=f"recipe name ({', '.join(sorted(RECIPES))}) or path of a YAML config")
    ap.add_argument("--load-path", required=True)
    ap.add_argument("--start-lr", type=float, required=True, help="learning rate of the base run at the checkpoint")
    ap.add_argument("--tokens", type=float, required=True, help="annealing budget in tokens")
    ap.add_argument("--name", required=True)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--mix", default=None)
    ap.add_argument("--read-location", default="/data")
    ap.add_argument("--data-glob", default=None)
    ap.add_argument("-o", "--output", required=True)
    args = ap.parse_args(argv)

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
    if args.mix is not None:
        from olmo_b200.data.named_data_mixes import resolve_mix

        raw.setdefault("data", {})["paths"] = resolve_mix(args.mix, args.read_location)
    elif args.data_glob is not None:
        raw.setdefault("data", {})["paths"] = "${path.glob:" + args.data_glob + "}"
    Path(args.output).write_text(f"# annealing run derived from {args.base}\n" + S.dump_yaml(raw))
    TrainConfig.load(args.output, validate_paths=False)  # the result must validate
    return raw


if __name__ == "__main__":
    main()
