#!/usr/bin/env python
"""Write a checkpoint in a sharded layout the reference implementation loads.

    scripts/export_sharded.py IN_DIR OUT_DIR [--world-size N] [--model-only]

``IN_DIR`` is any checkpoint this framework reads: unsharded (``model.pt`` / ``.safetensors``), its own flat-shard
format, or a reference sharded layout.  ``OUT_DIR`` receives the ``torch_new`` layout (``model_and_optim/`` in torch's
distributed-checkpoint format, ``train/rank*.pt``, ``config.yaml`` with ``sharded_checkpointer: torch_new``), which is
resharded by its reader, so it loads at any world size.  The inverse of ``scripts/unshard.py``; runs on one CPU process.
"""
from __future__ import annotations

import argparse
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch

from olmo_b200.checkpoint import build_sharded_checkpointer
from olmo_b200.checkpoint_compat import detect_layout, export_torch_new_checkpoint
from olmo_b200.config import ShardedCheckpointerType, TrainConfig

log = logging.getLogger(__name__)


def read_full_states(input_dir: Path, config: TrainConfig, model_only: bool):
    layout = detect_layout(input_dir)
    if layout != "unsharded":
        ckpt = build_sharded_checkpointer(config)
        return ckpt.unshard_checkpoint(input_dir, load_optimizer_state=not model_only, load_trainer_state=not model_only)
    if (input_dir / "model.safetensors").is_file():
        from olmo_b200.safetensors_util import safetensors_file_to_state_dict as load
        suffix = "safetensors"
    else:
        def load(path):
            return torch.load(path, map_location="cpu", weights_only=False)
        suffix = "pt"
    model = load(input_dir / f"model.{suffix}")
    optim = trainer = None
    if not model_only:
        optim = load(input_dir / f"optim.{suffix}") if (input_dir / f"optim.{suffix}").is_file() else None
        trainer = load(input_dir / f"train.{suffix}") if (input_dir / f"train.{suffix}").is_file() else None
    return model, optim, trainer


def main(input_dir, output_dir, world_size: int = 1, model_only: bool = False) -> Path:
    input_dir, output_dir = Path(input_dir), Path(output_dir)
    config = TrainConfig.load(input_dir / "config.yaml", validate_paths=False)
    model, optim, trainer = read_full_states(input_dir, config, model_only)
    out = export_torch_new_checkpoint(output_dir, model, optim, trainer, world_size=world_size)
    config.sharded_checkpointer = ShardedCheckpointerType.torch_new
    config.save(out / "config.yaml")
    log.info("wrote %s (%d tensors, optimizer state %s)", out, len(model), "included" if optim is not None else "left out")
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("input_dir")
    ap.add_argument("output_dir")
    ap.add_argument("--world-size", type=int, default=1, help="number of per-rank trainer-state files to write")
    ap.add_argument("--model-only", action="store_true")
    args = ap.parse_args()
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    main(args.input_dir, args.output_dir, world_size=args.world_size, model_only=args.model_only)
