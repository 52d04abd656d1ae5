#!/usr/bin/env python
"""Convert a sharded checkpoint into the unsharded layout (``model.pt``, ``optim.pt``, ``train.pt``, ``config.yaml``) that
both this framework and the reference load (reference: ``scripts/unshard.py:15-115``).  Runs offline on one CPU process.

The layout of the input directory is detected: this framework's flat-shard format, or the reference's ``torch_legacy``
(``rank*.pt`` holding ``ShardedTensor`` pickles), ``torch_new`` (``model_and_optim/``) and ``local`` (raw flat-parameter
pieces) layouts.  ``--type`` is checked against what is found, so a wrong guess is reported instead of misread."""
from __future__ import annotations

import argparse
import logging
import shutil
import sys
from pathlib import Path
from typing import Union

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch

from olmo_b200.checkpoint import build_sharded_checkpointer
from olmo_b200.config import ShardedCheckpointerType, TrainConfig
from olmo_b200.safetensors_util import state_dict_to_safetensors_file

logger = logging.getLogger(__name__)


def main(
    input_dir: Union[str, Path], output_dir: Union[str, Path], sharded_checkpoint_type: ShardedCheckpointerType = ShardedCheckpointerType.torch_legacy,
    model_only: bool = False, safe_tensors: bool = False, use_shared_mem_impl: bool = False,
) -> None:
    input_dir, output_dir = Path(input_dir), Path(output_dir)
    output_dir.mkdir(parents=True, exist_ok=True)
    config = TrainConfig.load(input_dir / "config.yaml", validate_paths=False)
    from olmo_b200.checkpoint_compat import detect_layout

    found = detect_layout(input_dir)
    if found not in ("flat_shard", str(getattr(sharded_checkpoint_type, "value", sharded_checkpoint_type))):
        logger.warning("--type says %s but %s holds a '%s' checkpoint; reading it as '%s'", sharded_checkpoint_type, input_dir, found, found)
    checkpointer = build_sharded_checkpointer(config, name=sharded_checkpoint_type, use_shared_mem_impl=use_shared_mem_impl)
    model_state, optim_state, trainer_state = checkpointer.unshard_checkpoint(
        input_dir, load_optimizer_state=not model_only, load_trainer_state=not model_only
    )

    def write(obj, stem: str) -> None:
        if safe_tensors:
            state_dict_to_safetensors_file(obj, output_dir / f"{stem}.safetensors")
        else:
            torch.save(obj, output_dir / f"{stem}.pt")
        logger.info("Saved %s state to %s", stem, output_dir)

    write(model_state, "model")
    if not model_only:
        write(optim_state, "optim")
        write(trainer_state, "train")
    shutil.copy(input_dir / "config.yaml", output_dir)


if __name__ == "__main__":
    ap = argparse.ArgumentParser(prog="unshard.py", description="Unshard sharded checkpoints on CPU")
    ap.add_argument("input_dir")
    ap.add_argument("output_dir")
    ap.add_argument("--type", choices=list(ShardedCheckpointerType), default=ShardedCheckpointerType.torch_legacy, type=ShardedCheckpointerType)
    ap.add_argument("--model-only", action="store_true")
    ap.add_argument("--safe-tensors", action="store_true")
    ap.add_argument("--use-legacy-shared-mem-impl", action="store_true", help="accepted for command-line compatibility; has no effect")
    a = ap.parse_args()
    logging.basicConfig(level=logging.INFO)
    main(a.input_dir, a.output_dir, a.type, a.model_only, a.safe_tensors, a.use_legacy_shared_mem_impl)
