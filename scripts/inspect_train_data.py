#!/usr/bin/env python
"""Show what a given rank saw at given training steps.  With ``data-indices/rank{R}.tsv.gz`` files (written when
``save_data_indices`` is on) the dataset indices are read back; otherwise the order is re-derived from the run's config
and seed, which is possible because the global order is a pure function of (seed, epoch, dataset size)
(reference: ``scripts/inspect_train_data.py``).

    python scripts/inspect_train_data.py RUN_DIR RANK STEP [STEP ...] [--world_size W] [--no_data_indices] [--ids]
                                         [--checkpoint_num N] [--mount weka:// /weka/] [--epoch E]

``--checkpoint_num N`` anchors the re-derivation at the trainer state saved with checkpoint ``stepN`` (its epoch and the number
of examples already consumed in that epoch), which is what makes steps after a restart, a change of batch size or an epoch
boundary come out right.  ``--mount URL DIR`` says that the run saw ``URL`` mounted at ``DIR``: data paths under ``DIR`` are
read from ``URL`` here.
"""
from __future__ import annotations

import argparse
import gzip
import sys
from pathlib import Path
from typing import Dict, Iterable, List, Optional

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.config import TrainConfig
from olmo_b200.data import IterableDataset, build_memmap_dataset
from olmo_b200.util import clean_opt, prepare_cli_environment


def indices_from_files(folder: Path, ranks: Optional[List[int]], steps: Iterable[int]) -> Dict[tuple, List[int]]:
    files = sorted((folder / "data-indices").glob("rank*.tsv.gz"))
    want = set(steps)
    out: Dict[tuple, List[int]] = {}
    for f in files:
        rank = int(f.name[len("rank") : -len(".tsv.gz")])
        if ranks is not None and rank not in ranks:
            continue
        with gzip.open(f, "rt") as fh:
            for line in fh:
                parts = line.rstrip("\n").split("\t")
                if parts and parts[0].isdigit() and int(parts[0]) in want:
                    out[(int(parts[0]), rank)] = [int(x) for x in parts[1:]]
    return out


def anchor_from_checkpoint(run: Path, step: int) -> Dict[str, int]:
    """Epoch, step and examples consumed in the epoch, from the trainer state saved with checkpoint ``step``."""
    import torch

    for candidate in (run / f"step{step}" / "train" / "rank0.pt", run / f"step{step}-unsharded" / "train.pt"):
        if candidate.is_file():
            state = torch.load(candidate, map_location="cpu", weights_only=False)
            seen = state.get("global_train_examples_seen_this_epoch", state.get("global_train_examples_seen", 0))
            return {"epoch": int(state.get("epoch") or 0), "step": int(state["global_step"]), "examples": int(seen)}
    raise SystemExit(f"no trainer state of step {step} under {run} (looked for step{step}/train/rank0.pt and step{step}-unsharded/train.pt)")


def remount(paths: Optional[List[str]], mounts: List[List[str]]) -> Optional[List[str]]:
    """Replace the mounted directory prefix of every path by the URL it was a mount of."""
    if not paths or not mounts:
        return paths
    out = []
    for path in paths:
        for url, folder in mounts:
            if str(path).startswith(folder):
                path = (url if url.endswith("/") else url + "/") + str(path)[len(folder):].lstrip("/")
                break
        out.append(path)
    return out


def indices_from_seed(cfg: TrainConfig, dataset, world_size: int, ranks: List[int], steps: Iterable[int], epoch: int = 0,
                      anchor: Optional[Dict[str, int]] = None) -> Dict[tuple, List[int]]:
    seed = cfg.data.seed if cfg.data.seed is not None else cfg.seed
    if anchor is not None:
        epoch = anchor["epoch"]
    order = IterableDataset(dataset, cfg.global_train_batch_size, seed=seed, epoch=epoch, shuffle=True, drop_last=cfg.data.drop_last,
                            world_size=1, rank=0, fs_local_rank=0).get_global_indices()
    per_rank = cfg.global_train_batch_size // world_size
    out = {}
    for step in steps:
        if anchor is None:
            start = (step - 1) * cfg.global_train_batch_size  # step N consumes the N-th global batch
        else:  # batches after the anchored checkpoint continue from the examples it had consumed
            if step <= anchor["step"]:
                raise SystemExit(f"step {step} is not after checkpoint step {anchor['step']}: pick an earlier --checkpoint_num")
            start = anchor["examples"] + (step - anchor["step"] - 1) * cfg.global_train_batch_size
        window = order[start : start + cfg.global_train_batch_size]
        for rank in ranks:
            out[(step, rank)] = [int(i) for i in window[rank::world_size][:per_rank]]
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("run_path")
    ap.add_argument("rank", type=int, help="-1 for all ranks")
    ap.add_argument("steps", nargs="+", type=int)
    ap.add_argument("--no_data_indices", action="store_false", dest="use_data_indices")
    ap.add_argument("--world_size", type=int, default=None)
    ap.add_argument("--epoch", type=int, default=0)
    ap.add_argument("--ids", action="store_true", help="print token ids instead of decoded text")
    ap.add_argument("--checkpoint_num", type=int, default=-1, help="step of the checkpoint whose trainer state anchors the data order")
    ap.add_argument("--mount", default=[], nargs=2, action="append", dest="mounts", metavar=("URL", "DIR"),
                    help="the run saw URL mounted at DIR, e.g. --mount weka:// /weka/")
    ap.add_argument("--save_overwrite", action="store_true", help="accepted for compatibility (nothing is written)")
    args = ap.parse_args(argv)
    prepare_cli_environment()
    run = Path(args.run_path)
    cfg = TrainConfig.load(run / "config.yaml", overrides=[clean_opt("--evaluators=[]")], validate_paths=False)
    cfg.data.paths = remount(cfg.data.paths, args.mounts)
    if cfg.data.datasets:
        cfg.data.datasets = {label: remount(list(group), args.mounts) for label, group in cfg.data.datasets.items()}
    dataset = build_memmap_dataset(cfg, cfg.data)
    if args.use_data_indices and (run / "data-indices").is_dir():
        found = indices_from_files(run, None if args.rank < 0 else [args.rank], args.steps)
    else:
        if args.world_size is None:
            raise SystemExit("--world_size is required when data indices are not available")
        ranks = list(range(args.world_size)) if args.rank < 0 else [args.rank]
        anchor = anchor_from_checkpoint(run, args.checkpoint_num) if args.checkpoint_num >= 0 else None
        found = indices_from_seed(cfg, dataset, args.world_size, ranks, args.steps, args.epoch, anchor=anchor)
    tokenizer = None
    if not args.ids:
        from olmo_b200.tokenizer import Tokenizer

        tokenizer = Tokenizer.from_train_config(cfg)
    for (step, rank), indices in sorted(found.items()):
        for i, index in enumerate(indices):
            ids = dataset[index]["input_ids"].tolist()
            shown = ids if tokenizer is None else tokenizer.decode(ids)
            print(f'[step={step}, rank={rank}, example={i}, index={index}] "{shown}"\n')
    return len(found)


if __name__ == "__main__":
    main()
