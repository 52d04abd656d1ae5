"""
Reference arm of ``bench.py``: the unmodified allenai/OLMo package installed under ``baseline/_ref`` (``pip install
--no-deps --target``), driven through its own public API on the same config and synthetic data as the main arm.

The path is the one ``scripts/train.py`` of the reference takes: ``TrainConfig`` → ``OLMo(cfg.model)`` on the meta
device → ``torch.distributed.fsdp.FullyShardedDataParallel`` with the model's own wrap policy and mixed precision →
``build_optimizer`` / ``build_scheduler`` → ``Trainer.train_step``.  None of this repository's models, kernels or
engine is imported here.  Packages the reference imports at module load but that are absent from this image
(omegaconf, boto3, cached_path, google-cloud-storage, torchmetrics, importlib_resources) are satisfied by the inert
stand-ins under ``baseline/shims``; they are never exercised because the config objects are built directly and the
run touches no remote storage and no evaluators.
"""
from __future__ import annotations

import os
import sys
import tempfile
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _unavailable(reason: str) -> dict:
    return {"impl": "reference", "unavailable": reason}


def run_reference(args, presets) -> dict:
    ref_root = HERE / "_ref"
    if not (ref_root / "olmo" / "model.py").is_file():
        return _unavailable("baseline/_ref is missing: install the reference there with pip --no-index --no-deps --target baseline/_ref <reference checkout>")
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(HERE / "shims"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")

    import torch

    if not torch.cuda.is_available():
        return _unavailable("no CUDA device")
    try:
        return _run(args, presets)
    except torch.cuda.OutOfMemoryError as e:  # report instead of crashing the driver's sequence
        return _unavailable(f"reference ran out of device memory on this config: {str(e)[:160]}")


def _run(args, presets) -> dict:
    import torch
    import torch.distributed as dist
    from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

    from olmo.config import (  # the reference's own classes
        ActivationCheckpointingStrategy, DistributedStrategy, FSDPConfig, FSDPPrecision, FSDPWrapStrategy, InitFnType,
        LayerNormType, ModelConfig, OptimizerConfig, OptimizerType, SchedulerConfig, SchedulerType, SchedulerUnits,
        ShardingStrategy, SpeedMonitorConfig, TrainConfig,
    )
    from olmo.model import OLMo
    from olmo.optim import build_optimizer, build_scheduler
    from olmo.torch_util import get_default_device, seed_all
    from olmo.train import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("LOCAL_RANK", "0")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda")
    dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"

    ps = presets[args.model]
    olmo2 = ps["flavour"] == "olmo2"
    seq = args.seq_len
    model_cfg = ModelConfig(
        d_model=ps["d_model"], n_heads=ps["n_heads"], n_layers=ps["n_layers"], mlp_hidden_size=ps["mlp_hidden_size"],
        weight_tying=False, alibi=False, rope=True, rope_theta=500000 if olmo2 else 10000, flash_attention=True,
        attention_dropout=0.0, include_bias=False, layer_norm_type=LayerNormType.rms if olmo2 else LayerNormType.default,
        layer_norm_with_affine=olmo2, layer_norm_eps=1e-6 if olmo2 else 1e-5, bias_for_layer_norm=False,
        attention_layer_norm=olmo2, attention_layer_norm_with_affine=olmo2, norm_after=olmo2, residual_dropout=0.0,
        embedding_dropout=0.0, max_sequence_length=seq, vocab_size=100278 if olmo2 else 50280,
        embedding_size=100352 if olmo2 else 50304, eos_token_id=100257 if olmo2 else 50279, pad_token_id=100277 if olmo2 else 1,
        init_device="meta", init_fn=InitFnType.normal if olmo2 else InitFnType.mitchell, init_std=0.02,
        init_cutoff_factor=3 if olmo2 else None, clip_qkv=None if olmo2 else 8.0,
    )
    device_batch = args.device_batch or max(ps["microbatch"], min(32, ps["global_batch"] // 8))  # same default as the main arm
    sharding = ShardingStrategy[getattr(args, "sharding", "FULL_SHARD")]
    ac = None if args.activation_checkpointing in (None, "none") else ActivationCheckpointingStrategy(args.activation_checkpointing)
    cfg = TrainConfig(
        run_name=f"bench-ref-{args.model}", model=model_cfg,
        optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=3e-4, weight_decay=0.1, eps=1e-8, betas=(0.9, 0.95),
                                  decay_norm_and_bias=True, decay_embeddings=False),
        scheduler=SchedulerConfig(name=SchedulerType.cosine_with_warmup, units=SchedulerUnits.tokens, t_warmup=8388608000, t_max=5e12,
                                  alpha_f=0.1, warmup_min_lr=0.0),
        global_train_batch_size=device_batch * world, device_train_microbatch_size=ps["microbatch"], precision="amp_bf16",
        distributed_strategy=DistributedStrategy.fsdp,
        fsdp=FSDPConfig(sharding_strategy=sharding, wrapping_strategy=FSDPWrapStrategy.by_block_and_size,
                        precision=FSDPPrecision.mixed,
                        hybrid_sharding_num_model_replicas=(args.replicas or 2) if sharding == ShardingStrategy.HYBRID_SHARD else None),
        max_grad_norm=1.0, softmax_auxiliary_loss=True, auxiliary_loss_multiplier=1e-5, fused_loss=True,
        save_folder=tempfile.mkdtemp(prefix="olmo_ref_bench_"), save_overwrite=True, save_data_indices=False,
        max_duration=10**9, console_log_interval=10**9, speed_monitor=SpeedMonitorConfig(window_size=1),
        activation_checkpointing=ac,
    )
    # the same derived fields scripts/train.py fills in
    cfg.model.precision = cfg.precision
    cfg.device_train_batch_size = cfg.global_train_batch_size // world
    cfg.device_train_grad_accum = cfg.device_train_batch_size // cfg.device_train_microbatch_size

    seed_all(cfg.seed)
    olmo_model = OLMo(cfg.model)
    flops_per_token = olmo_model.num_fwd_flops + olmo_model.num_bck_flops  # read before sharding: FSDP leaves local shards only
    olmo_model.set_activation_checkpointing(cfg.activation_checkpointing)
    wrap_policy = olmo_model.get_fsdp_wrap_policy(cfg.fsdp.wrapping_strategy)

    def dummy_init_fn(module: torch.nn.Module) -> None:
        module.to_empty(device=get_default_device())

    device_mesh = None
    if sharding in (ShardingStrategy.HYBRID_SHARD, ShardingStrategy._HYBRID_SHARD_ZERO2):
        # the 2-D mesh scripts/train.py of the reference builds: (replicas, ranks per replica)
        from torch.distributed.device_mesh import init_device_mesh

        replicas = cfg.fsdp.hybrid_sharding_num_model_replicas or 2
        device_mesh = init_device_mesh("cuda", (replicas, world // replicas))
    dist_model = FSDP(
        olmo_model, sharding_strategy=cfg.fsdp.sharding_strategy, mixed_precision=cfg.fsdp_precision,
        auto_wrap_policy=wrap_policy, use_orig_params=cfg.fsdp.use_orig_params, limit_all_gathers=True,
        device_id=local_rank, param_init_fn=dummy_init_fn, device_mesh=device_mesh,
    )
    olmo_model.reset_parameters()
    optim = build_optimizer(cfg, dist_model)
    scheduler = build_scheduler(cfg)

    trainer = Trainer(
        cfg=cfg, epoch=cfg.epoch, model=olmo_model, dist_model=dist_model, optim=optim, scheduler=scheduler,
        train_loader=None, device=device, evaluators=[], indices_file=None,  # type: ignore[arg-type]
    )

    # identical synthetic data: (seed, index) -> tokens, generated by the same numpy recipe as the main arm
    import numpy as np

    def instance(index: int) -> "torch.Tensor":
        rng = np.random.Generator(np.random.PCG64([cfg.seed, index]))
        ids = rng.integers(0, cfg.model.vocab_size, size=seq, dtype=np.int64)
        ids[rng.random(seq) < 1.0 / 256] = cfg.model.eos_token_id
        return torch.from_numpy(ids)

    def host_batch(step: int) -> "torch.Tensor":
        out = torch.empty((device_batch, seq), dtype=torch.int64, pin_memory=True)
        first = (step * world + rank) * device_batch
        for j in range(device_batch):
            out[j] = instance((first + j) % (1 << 20))
        return out

    host_batches = [host_batch(s) for s in range(min(args.warmup + 2 * args.steps + 1, 4))]
    dev_batches = [b.to(device) for b in host_batches]

    def step(i: int, from_host: bool) -> float:
        ids = host_batches[i % len(host_batches)] if from_host else dev_batches[i % len(dev_batches)]
        trainer.global_step += 1
        trainer.global_train_tokens_seen += device_batch * world * seq
        return trainer.train_step({"input_ids": ids}, reduce_global_loss=False)["train/CrossEntropyLoss"]

    def barrier() -> None:
        dist.barrier()
        torch.cuda.synchronize()

    sys.path.insert(0, str(HERE.parent))
    from bench import ClockSampler, bench_config  # timing / reporting helpers only

    loss = float("nan")
    for i in range(args.warmup):
        loss = step(i, False)
    sampler = ClockSampler(local_rank)
    barrier()
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        loss = step(args.warmup + i, False)
    ev1.record()
    barrier()
    clocks = sampler.stop()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = t.item() / args.steps

    e2e = None
    if not args.no_e2e:
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            loss = step(args.warmup + args.steps + i, True)
        barrier()
        wall = torch.tensor([time.perf_counter() - t0], device=device, dtype=torch.float64)
        dist.all_reduce(wall, op=dist.ReduceOp.MAX)
        e2e = {
            "value": device_batch * world * seq * args.steps / wall.item(), "unit": "tokens/s",
            "h2d_bytes_per_step": device_batch * seq * 8, "d2h_bytes_per_step": 16, "ms_per_step": wall.item() * 1e3 / args.steps,
        }

    tokens_per_step = device_batch * world * seq
    value = tokens_per_step / (ms_per_step / 1e3)
    result = {
        "metric": f"tokens_per_second ({'OLMo-2' if olmo2 else 'OLMo-1'} training, whole job; FSDP {sharding.name}, device-timed, max over ranks)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic seeded uniform tokens with EOS boundaries; random-init weights", "impl": "reference",
        "tokens_per_second_per_gpu": value / world, "mfu_nominal_2250tf": value / world * flops_per_token / 2.25e15,
        "flops_per_token": flops_per_token, "final_loss": loss,
        "config": bench_config(args, ps, device_batch, world, cfg.device_train_grad_accum),
        "implementation": {"engine": f"torch FSDP1 {sharding.name} (NCCL), cuBLAS, flash-attn"},
        "clocks": clocks, "e2e": e2e, "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9,
    }
    dist.destroy_process_group()
    return result if rank == 0 else {}
