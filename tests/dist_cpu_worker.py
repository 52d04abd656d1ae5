"""Worker for the multi-process CPU tests (gloo).  One scenario per invocation; launched by ``test_dist_cpu.py`` either
directly (one rank) or through ``python -m torch.distributed.run`` (several ranks)."""
import argparse
import datetime
import os
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def build(args, world: int, save_folder: str):
    from olmo_b200.config import (
        DistributedStrategy, FSDPConfig, FSDPPrecision, FSDPWrapStrategy, LayerNormType, ModelConfig, OptimizerConfig,
        OptimizerType, SchedulerConfig, SchedulerType, ShardingStrategy, TrainConfig,
    )
    from olmo_b200.launch import build_trainer, derive_batch_sizes

    model = ModelConfig(
        d_model=64, n_heads=4, n_layers=3, mlp_hidden_size=256, weight_tying=False, rope=True, flash_attention=False,
        attention_dropout=0.0, residual_dropout=0.0, embedding_dropout=0.0, include_bias=False, layer_norm_type=LayerNormType.rms,
        layer_norm_with_affine=True, attention_layer_norm=True, norm_after=True, max_sequence_length=32, vocab_size=250,
        embedding_size=256, eos_token_id=249, pad_token_id=249, init_device="meta", init_std=0.05,
    )
    cfg = TrainConfig(
        model=model,
        optimizer=OptimizerConfig(name=OptimizerType[args.optimizer], learning_rate=2e-3, eps=1e-8, weight_decay=0.1),
        scheduler=SchedulerConfig(name=SchedulerType.constant), precision="fp32",
        distributed_strategy=DistributedStrategy.fsdp if world > 1 or args.force_fsdp else DistributedStrategy.single,
        fsdp=FSDPConfig(sharding_strategy=ShardingStrategy[args.strategy], wrapping_strategy=FSDPWrapStrategy[args.wrap],
                        precision=FSDPPrecision.pure, hybrid_sharding_num_model_replicas=args.replicas),
        global_train_batch_size=8, device_train_microbatch_size=2, max_grad_norm=1.0, save_folder=save_folder, save_overwrite=True,
        save_data_indices=False, console_log_interval=1000, max_duration=100, softmax_auxiliary_loss=True, time_limit=args.time_limit,
        sharded_checkpointer=args.checkpointer,
    )
    derive_batch_sizes(cfg, world)
    from torch.utils.data import DataLoader

    from olmo_b200.data import DataCollator, IterableDataset, SyntheticTokenDataset

    ds = SyntheticTokenDataset(256, 32, 16, 249, seed=1, mean_doc_len=0)
    it = IterableDataset(ds, cfg.global_train_batch_size, seed=0, world_size=world, rank=int(os.environ.get("RANK", "0")), fs_local_rank=0, num_threads=0)
    loader = DataLoader(it, batch_size=cfg.device_train_batch_size, collate_fn=DataCollator.from_train_config(cfg))
    trainer = build_trainer(cfg, device=torch.device("cpu"), train_loader=loader, with_evaluators=False)
    return cfg, trainer


def run_steps(trainer, cfg, n, batches):
    out = []
    for _ in range(n):
        trainer.global_step += 1
        trainer.global_train_examples_seen_this_epoch += cfg.global_train_batch_size
        trainer.global_train_tokens_seen += cfg.global_train_batch_size * cfg.model.max_sequence_length
        m = trainer.train_step(next(batches))
        out.append({"loss": m["train/CrossEntropyLoss"], "norm": float(m.get("optim/total_grad_norm", 0.0))})
    return out


def full_state(trainer):
    eng = trainer.dist_model.engine
    return eng.full_model_state_dict(rank0_only=True, cpu=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("scenario", choices=["train", "save", "restore", "cancel", "lost_rank", "save_crash"])
    ap.add_argument("--out", required=True)
    ap.add_argument("--work", required=True)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--strategy", default="FULL_SHARD")
    ap.add_argument("--wrap", default="by_block")
    ap.add_argument("--replicas", type=int, default=None)
    ap.add_argument("--optimizer", default="adamw")
    ap.add_argument("--checkpointer", default="olmo_core")
    ap.add_argument("--force-fsdp", action="store_true")
    ap.add_argument("--time-limit", type=float, default=None)
    ap.add_argument("--load", default=None)
    ap.add_argument("--pg-timeout", type=float, default=60.0)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=args.pg_timeout))
    torch.manual_seed(0)
    cfg, trainer = build(args, world, args.work)
    batches = iter(trainer.train_loader)
    result = {"world": world}

    if args.scenario == "train":
        result["steps"] = run_steps(trainer, cfg, args.steps, batches)
        state = full_state(trainer)
        if rank == 0:
            result["state"] = state
    elif args.scenario == "save":
        result["steps"] = run_steps(trainer, cfg, args.steps, batches)
        path, _ = trainer.save_checkpoint()
        upath, _ = trainer.save_unsharded_checkpoint()
        result["sharded"], result["unsharded"] = str(path), str(upath)
        state = full_state(trainer)
        if rank == 0:
            result["state"] = state
        result["next"] = run_steps(trainer, cfg, 1, batches)
    elif args.scenario == "restore":
        trainer.restore_checkpoint(args.load)
        result["global_step"] = trainer.global_step
        state = full_state(trainer)
        if rank == 0:
            result["state"] = state
        batches = iter(trainer.train_loader)
        result["next"] = run_steps(trainer, cfg, 1, batches)
    elif args.scenario == "save_crash":
        # a good checkpoint at step 2; during the save at step 3 the last rank dies after its shards are written and
        # before the temporary folder is renamed (host-side fault: the process exits, nothing is in flight on a device)
        run_steps(trainer, cfg, 2, batches)
        good, _ = trainer.save_checkpoint()
        run_steps(trainer, cfg, 1, batches)
        from olmo_b200 import checkpoint as ckpt

        if rank == world - 1:
            ckpt.Checkpointer._save_config = lambda self, *a, **k: os._exit(17)  # called last inside the temporary folder
        if rank == 0:
            torch.save({"good": str(good), "world": world}, args.out)
        try:
            trainer.save_checkpoint()
        except Exception as e:  # noqa: BLE001 - the surviving ranks must get an error from their next collective
            torch.save({"error": type(e).__name__}, f"{args.out}.rank{rank}")
            os._exit(3)
        os._exit(0)
    elif args.scenario == "cancel":
        # rank 0 alone owns the clock; every rank must learn of the cancellation at the same step
        trainer._start_time = time.time() - (10_000.0 if rank == 0 else 0.0)
        stopped_at = None
        for step in range(1, 6):
            run_steps(trainer, cfg, 1, batches)
            trainer.cancelled, extra = trainer.check_if_cancelled()
            if trainer.cancelled:
                stopped_at = step
                break
        result["stopped_at"] = stopped_at
    elif args.scenario == "lost_rank":
        # the last rank leaves between steps (nothing in flight); the others must get an error, not a hang
        run_steps(trainer, cfg, 1, batches)
        dist.barrier()
        if rank == world - 1:
            torch.save({"left": True}, f"{args.out}.rank{rank}")
            os._exit(0)
        t0 = time.time()
        try:
            run_steps(trainer, cfg, 1, batches)
            result["error"] = None
        except Exception as e:  # noqa: BLE001 - any collective failure is what we are after
            result["error"] = type(e).__name__
        result["waited"] = time.time() - t0
        torch.save(result, f"{args.out}.rank{rank}")
        os._exit(0)

    if rank == 0:
        torch.save(result, args.out)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
