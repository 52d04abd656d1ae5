#!/usr/bin/env python
"""Replay the training data order of a config without a model and write the batches to ``.npy`` files
(``{field}-{first:07d}-{last:07d}.npy``, 1000 batches per file by default); used to audit or pre-materialise exactly what
a run will see (reference: ``scripts/run_dataloader.py``).

    python scripts/run_dataloader.py CONFIG.yaml -o OUT_DIR [--batches N] [--world-size W --rank R] [--a.b=c ...]
"""
import argparse
import logging
import sys
from pathlib import Path
from typing import Dict

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np
from torch.utils.data import DataLoader

from olmo_b200.config import TrainConfig
from olmo_b200.data import DataCollator, IterableDataset, build_memmap_dataset
from olmo_b200.launch import derive_batch_sizes
from olmo_b200.util import clean_opt, prepare_cli_environment

log = logging.getLogger("run_dataloader")


def main(cfg: TrainConfig, output_dir: Path, world_size: int, rank: int, max_batches=None, batches_per_file: int = 1000) -> int:
    derive_batch_sizes(cfg, world_size)
    dataset = build_memmap_dataset(cfg, cfg.data, include_instance_metadata=False)
    seed = cfg.data.seed if cfg.data.seed is not None else cfg.seed
    workers = cfg.data.num_workers
    loader = DataLoader(
        IterableDataset(dataset, cfg.global_train_batch_size, seed=seed + (cfg.epoch or 0), shuffle=True, drop_last=cfg.data.drop_last,
                        world_size=world_size, rank=rank, fs_local_rank=0, work_dir=None),
        batch_size=cfg.device_train_batch_size, drop_last=cfg.data.drop_last,
        collate_fn=DataCollator(pad_direction=cfg.data.pad_direction, pad_token_id=cfg.model.pad_token_id),
        num_workers=workers, pin_memory=False, prefetch_factor=None if workers == 0 else cfg.data.prefetch_factor,
        persistent_workers=False, timeout=cfg.data.timeout,
    )
    small_vocab = (cfg.model.embedding_size or cfg.model.vocab_size) <= 2**16
    pending: Dict[str, list] = {}
    first = written = 0

    def flush(upto: int) -> None:
        nonlocal first
        for name, chunks in pending.items():
            np.save(output_dir / f"{name}-{first:07d}-{upto:07d}.npy", np.stack(chunks))
        pending.clear()
        first = upto

    for number, batch in enumerate(loader):
        if max_batches is not None and number >= max_batches:
            break
        for name, value in batch.items():
            if not hasattr(value, "numpy"):
                continue
            arr = value.numpy()
            if name == "input_ids":
                arr = arr.astype(np.uint16 if small_vocab else np.uint32)
            pending.setdefault(name, []).append(arr)
        written = number + 1
        if written - first >= batches_per_file:
            flush(written)
    if pending:
        flush(written)
    log.info("wrote %d batches to %s", written, output_dir)
    return written


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config_file")
    ap.add_argument("-o", required=True, help="output directory")
    ap.add_argument("--batches", type=int, default=None)
    ap.add_argument("--batches-per-file", type=int, default=1000)
    ap.add_argument("--world-size", type=int, default=1)
    ap.add_argument("--rank", type=int, default=0)
    args, rest = ap.parse_known_args()
    prepare_cli_environment()
    out = Path(args.o)
    out.mkdir(parents=True, exist_ok=True)
    overrides = ["save_folder=runs/"] + [clean_opt(s) for s in rest]
    main(TrainConfig.load(args.config_file, overrides), out, args.world_size, args.rank, args.batches, args.batches_per_file)
