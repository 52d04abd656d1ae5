#!/usr/bin/env python
"""
Training entry point:  ``[torchrun ...] scripts/train.py CONFIG.yaml [--dotted.key=value ...]``

Mirrors the command line of the reference's ``scripts/train.py:382-436``: one process per GPU under ``torchrun``
(NCCL for collectives that are not served by peer memory, Gloo on CPU), a YAML config with dotted overrides, optional
resume from the latest checkpoint, a pre-train checkpoint self-test, then ``Trainer.fit()``.
"""
from __future__ import annotations

import logging
import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from olmo_b200.config import CheckpointType, DistributedStrategy, TrainConfig
from olmo_b200.exceptions import OLMoCliError, OLMoConfigurationError
from olmo_b200.launch import build_trainer, derive_batch_sizes
from olmo_b200.optim import BoltOnWarmupScheduler
from olmo_b200.torch_util import barrier, get_global_rank, get_local_rank, peak_gpu_memory, seed_all
from olmo_b200.util import add_cached_path_clients, clean_opt, find_latest_checkpoint, log_extra_field, prepare_cli_environment

log = logging.getLogger("train")


def main(cfg: TrainConfig) -> None:
    if cfg.run_name is None:
        raise OLMoConfigurationError("--run_name is required")
    log_extra_field("run_name", cfg.run_name)
    if (cfg.reset_optimizer_state or cfg.reset_trainer_state) and cfg.load_path is None:
        log.warning("You want to reset the optimizer or trainer state, but we're not loading from the checkpoint. The setting has no effect.")
    barrier()

    if torch.cuda.is_available():
        torch.cuda.set_device(f"cuda:{get_local_rank()}")
        device = torch.device("cuda", get_local_rank())
    else:
        device = torch.device("cpu")
    if cfg.distributed_strategy == DistributedStrategy.single:
        device = cfg.single.get_device()

    derive_batch_sizes(cfg)
    if cfg.optimizer.no_decay_norm_and_bias is not None:
        log.warning("`no_decay_norm_and_bias` is deprecated; it overrides `decay_norm_and_bias` and `decay_embeddings`.")
        cfg.optimizer.decay_norm_and_bias = not cfg.optimizer.no_decay_norm_and_bias
        cfg.optimizer.decay_embeddings = not cfg.optimizer.no_decay_norm_and_bias
        cfg.optimizer.no_decay_norm_and_bias = None

    if get_global_rank() == 0:
        if cfg.data.paths is not None and len(cfg.data.paths) < 50:
            log.info("Configuration:\n%s", cfg)
        if not cfg.dry_run and (cfg.load_path is None or Path(cfg.load_path).parent != Path(cfg.save_folder)):
            save_path = Path(cfg.save_folder) / "config.yaml"
            if save_path.is_file() and not cfg.save_overwrite:
                raise OLMoConfigurationError(f"{save_path} already exists, use --save_overwrite to overwrite")
            log.info("Saving config to %s", save_path)
            save_path.parent.mkdir(exist_ok=True, parents=True)
            cfg.save(save_path)
    barrier()

    if cfg.wandb is not None and (get_global_rank() == 0 or not cfg.wandb.rank_zero_only):
        import wandb

        wandb_dir = Path(cfg.save_folder) / "wandb"
        wandb_dir.mkdir(parents=True, exist_ok=True)
        wandb.init(
            dir=str(wandb_dir), project=cfg.wandb.project, entity=cfg.wandb.entity, group=cfg.wandb.group, name=cfg.wandb.name,
            tags=cfg.wandb.tags, config=cfg.asdict(exclude=["wandb"]),
        )
    barrier()
    seed_all(cfg.seed)

    log.info("Building model, engine, optimizer and data loader...")
    with build_trainer(cfg, device=device) as trainer:
        log.info("Peak GPU Memory (MB) after setup: %d", int(peak_gpu_memory() or 0))
        if cfg.try_load_latest_save:
            if (Path(cfg.save_folder) / "latest-unsharded").exists():
                cfg.load_path = str(Path(cfg.save_folder) / "latest-unsharded")
            elif (Path(cfg.save_folder) / "latest").exists():
                cfg.load_path = str(Path(cfg.save_folder) / "latest")
            elif (latest := find_latest_checkpoint(cfg.save_folder)) is not None:
                cfg.load_path = str(latest)
            elif cfg.remote_save_folder is not None and (latest := find_latest_checkpoint(cfg.remote_save_folder)) is not None:
                cfg.load_path = str(latest)
            log.info("Resuming from %s", cfg.load_path) if cfg.load_path else log.info("No checkpoint to resume from; starting fresh")

        if not cfg.dry_run and not cfg.no_pre_train_checkpoint and cfg.load_path is None:
            kind = CheckpointType.sharded if cfg.distributed_strategy == DistributedStrategy.fsdp else CheckpointType.unsharded
            log.info("Saving pre-train checkpoint...")
            path, local = trainer.save_checkpoint(checkpoint_type=kind)
            log.info("Checkpoint saved to %s; restoring it as a self-test...", path)
            trainer.restore_checkpoint(local or path, checkpoint_type=kind)
            log.info("Checkpoint successfully loaded")
            if cfg.save_interval_ephemeral is None and cfg.save_num_checkpoints_to_keep != 0:
                pass  # kept as step0
            else:
                trainer.remove_checkpoint(checkpoint_type=kind)

        if cfg.load_path is not None:
            log.info("Loading checkpoint from %s...", cfg.load_path)
            trainer.restore_checkpoint(
                cfg.load_path, load_optimizer_state=not cfg.reset_optimizer_state, load_trainer_state=not cfg.reset_trainer_state,
                sharded_checkpointer=cfg.load_path_sharded_checkpointer,
            )
            log.info("Checkpoint successfully loaded")
            if cfg.reset_optimizer_state and not cfg.reset_trainer_state:
                # the optimizer restarts cold: re-warm the LR so that it meets the original curve
                trainer.scheduler = BoltOnWarmupScheduler.wrap(
                    trainer.scheduler, trainer.global_step, int(trainer.global_step + cfg.scheduler.t_warmup)
                )
        if cfg.force_save_unsharded and cfg.distributed_strategy != DistributedStrategy.single:
            log.info("Saving unsharded checkpoint...")
            path, _ = trainer.save_checkpoint(checkpoint_type=CheckpointType.unsharded)
            log.info("Unsharded checkpoint saved to %s", path)

        if not cfg.dry_run:
            log.info("Starting training...")
            trainer.fit()
            log.info("Training complete")
        else:
            log.info("Dry run complete")


def init_distributed() -> None:
    """Join the job's process group when launched by torchrun; a bare ``python`` launch stays single-process."""
    if "RANK" not in os.environ or int(os.environ.get("WORLD_SIZE", "1")) < 1:
        return
    if torch.cuda.is_available():
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(minutes=30), device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("gloo", timeout=timedelta(minutes=30))


if __name__ == "__main__":
    if len(sys.argv) < 2 or sys.argv[1] in ("-h", "--help"):
        print(f"{(__doc__ or '').strip()}\n\nEvery key of the configuration (olmo_b200/config.py: TrainConfig) can be overridden, for example\n"
              "  --run_name=NAME --save_folder=DIR --load_path=DIR_OR_URL --try_load_latest_save --model.n_layers=16\n"
              "  --optimizer.learning_rate=3e-4 --global_train_batch_size=1024 --device_train_microbatch_size=2\n"
              "  --fsdp.sharding_strategy=FULL_SHARD|HYBRID_SHARD|NO_SHARD --distributed_strategy=fsdp|ddp|single")
        raise SystemExit(0 if len(sys.argv) >= 2 else 2)
    try:
        mp.set_start_method("spawn", force=True)
    except RuntimeError as e:
        print(f"failed to set multiprocessing start method: {e}")
    init_distributed()
    prepare_cli_environment()
    add_cached_path_clients()
    try:
        yaml_path, overrides = sys.argv[1], sys.argv[2:]
    except IndexError:
        raise OLMoCliError(f"Usage: {sys.argv[0]} [CONFIG_PATH] [OPTIONS]")
    config = TrainConfig.load(yaml_path, [clean_opt(s) for s in overrides])
    if not torch.cuda.is_available() and "RANK" not in os.environ:
        config.distributed_strategy = DistributedStrategy.single  # the only strategy that needs no process group
    main(config)
    if dist.is_initialized():
        dist.destroy_process_group()
