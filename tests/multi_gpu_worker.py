"""Worker for the multi-GPU tests: trains a small OLMo-2 style model for a few steps on WORLD_SIZE ranks and lets rank 0
save the full fp32 weights.  Launched with ``python -m torch.distributed.run`` by ``test_multi_gpu.py``."""
import argparse
import os
import sys
import tempfile
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--global-batch", type=int, default=8)
    ap.add_argument("--fused-comm", type=int, default=1)
    ap.add_argument("--strategy", default="FULL_SHARD")
    ap.add_argument("--schedule", default="resident", choices=["resident", "sharded", "auto"])
    ap.add_argument("--comm-ctas", type=int, default=0, help="0: communication warps in every GEMM CTA; n > 0: n CTAs set aside")
    ap.add_argument("--layers", type=int, default=3)
    ap.add_argument("--replicas", type=int, default=None)
    ap.add_argument("--activation-checkpointing", default=None)
    ap.add_argument("--resume-at", type=int, default=0, help="after this many steps: save a sharded checkpoint, wipe the live state, restore")
    ap.add_argument("--ckpt-dir", default=None, help="folder shared by all ranks for --resume-at")
    args = ap.parse_args()
    os.environ["OLMO_B200_FUSED_COMM"] = str(args.fused_comm)
    os.environ["OLMO_B200_SCHEDULE"] = args.schedule
    os.environ["OLMO_B200_COMM_CTAS"] = str(args.comm_ctas)
    os.environ["OLMO_B200_RS_CTAS"] = str(2 * args.comm_ctas)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

    from olmo_b200 import ops
    from olmo_b200.config import (
        DistributedStrategy, FSDPConfig, FSDPPrecision, FSDPWrapStrategy, LayerNormType, ModelConfig, OptimizerConfig,
        OptimizerType, SchedulerConfig, SchedulerType, ShardingStrategy, TrainConfig,
    )
    from olmo_b200.launch import build_model_and_engine, derive_batch_sizes
    from olmo_b200.optim import build_optimizer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)

    model = ModelConfig(
        d_model=256, n_heads=2, n_layers=args.layers, mlp_hidden_size=1024, weight_tying=False, rope=True, rope_theta=500000,
        flash_attention=True, attention_dropout=0.0, residual_dropout=0.0, embedding_dropout=0.0, include_bias=False,
        layer_norm_type=LayerNormType.rms, layer_norm_with_affine=True, layer_norm_eps=1e-6, bias_for_layer_norm=False,
        attention_layer_norm=True, norm_after=True, max_sequence_length=256, vocab_size=500, embedding_size=512,
        eos_token_id=499, pad_token_id=499, init_device="meta", init_std=0.05,
    )
    cfg = TrainConfig(
        model=model, optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=1e-3, eps=1e-8, weight_decay=0.1),
        scheduler=SchedulerConfig(name=SchedulerType.constant), precision="amp_bf16",
        distributed_strategy=DistributedStrategy.fsdp,
        fsdp=FSDPConfig(sharding_strategy=ShardingStrategy[args.strategy], wrapping_strategy=FSDPWrapStrategy.by_block_and_size, precision=FSDPPrecision.mixed,
                        hybrid_sharding_num_model_replicas=args.replicas),
        global_train_batch_size=args.global_batch, device_train_microbatch_size=2, max_grad_norm=1.0, save_folder=tempfile.mkdtemp(),
    )
    derive_batch_sizes(cfg, world)
    dist_model = build_model_and_engine(cfg, device)
    engine = dist_model.engine
    assert engine.fused
    if world > 1 and args.fused_comm:
        assert engine.comm is not None, "peer-memory collectives should be active"
        if args.replicas:
            assert engine.num_replicas == args.replicas and engine.comm.replicas == args.replicas
    if world > 1 and args.fused_comm and args.strategy == "FULL_SHARD":
        assert engine.schedule == args.schedule, (engine.schedule, args.schedule)
        if args.schedule == "sharded":
            assert sum(u.streamed for u in engine.units) == args.layers and engine.comm.full_slots is not None
    optim = build_optimizer(cfg, dist_model)

    from olmo_b200.config import ActivationCheckpointingStrategy

    ac = ActivationCheckpointingStrategy(args.activation_checkpointing) if args.activation_checkpointing else None
    db = cfg.device_train_batch_size
    gen = torch.Generator().manual_seed(1234)
    all_ids = torch.randint(0, 500, (args.steps, args.global_batch, 256), generator=gen)
    norms = []
    for step in range(args.steps):
        engine.zero_grad()
        mine = all_ids[step, rank * db : (rank + 1) * db].to(device)
        mbs = mine.split(cfg.device_train_microbatch_size)
        for i, mb in enumerate(mbs):
            labels = torch.nn.functional.pad(mb[:, 1:], (0, 1), value=-100)
            engine.train_microbatch(mb, labels, float(mine.numel()), z_mult=1e-4, is_last=i == len(mbs) - 1, ac_strategy=ac)
        m = optim.clip_grads_and_collect_metrics(step + 1, collect_param_metrics=False, process_group=engine.process_group)
        norms.append(float(m["total_grad_norm"]))
        optim.step()
        if args.resume_at and step + 1 == args.resume_at:
            # a resume inside one process: checkpoint, destroy what the checkpoint has to bring back, restore
            from olmo_b200.checkpoint import build_sharded_checkpointer

            cfg.save_overwrite = True
            ckpt = build_sharded_checkpointer(cfg)
            folder = os.path.join(args.ckpt_dir, "step")
            ckpt.save_checkpoint(folder, dist_model, optim, {"global_step": step + 1})
            for u in engine.units:
                u.master.fill_(7.0)
            for st in optim.state.values():
                for v in st.values():
                    if torch.is_tensor(v):
                        v.zero_()
            engine.params_changed()
            trainer_state = ckpt.restore_checkpoint(folder, dist_model, optim)
            assert trainer_state["global_step"] == step + 1
    ops.check_status()
    state = engine.full_model_state_dict(rank0_only=True, cpu=True)
    # the fused evaluation pass and the module-level forward (streamed units gathered for its duration) must agree
    probe = all_ids[0, :2].to(device)
    ce_sum, n_tok = engine.eval_loss(probe, torch.nn.functional.pad(probe[:, 1:], (0, 1), value=-100))
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits = dist_model(probe).logits
    ce_module = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), probe[:, 1:].reshape(-1), reduction="sum")
    if rank == 0:
        torch.save({"state": state, "norms": norms, "eval_ce": float(ce_sum) / float(n_tok), "module_ce": float(ce_module) / float(n_tok)}, args.out)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
