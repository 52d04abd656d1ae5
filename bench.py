#!/usr/bin/env python
"""
Headline benchmark: OLMo-2 training throughput (tokens/s over the whole job, plus per-GPU and MFU) on N B200s of
one node, synthetic seeded token data, random-init weights, bf16 compute with fp32 master weights and reduction.

    python bench.py --gpus 1 --steps 2 --warmup 3
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 --master-port 29500 \
        bench.py --gpus 8 --steps 2 --warmup 3
    python bench.py --impl reference ...        # the unmodified reference (baseline/_ref) on the same config

Per GPU the work is fixed (weak scaling): ``--device-batch`` sequences of ``seq_len`` tokens per optimizer step, split
into micro-batches of the model's official size (2 for the 7B preset), so the global batch is ``N × device_batch``.
The official run accumulates 64 micro-batches per GPU and step (1024 sequences over 8 GPUs, ``--device-batch 128``:
26 s per step here, 52 s for the reference arm); the default is 32 sequences (16 micro-batches) so that a run with
many timed steps still finishes in minutes.  Throughput hardly depends on it, because only the once-per-step work
(optimizer, gather, reduce-scatter; about 40 ms) is amortised differently; both figures are given in the repository's
design notes.

Two measurements are reported: ``value`` times K optimizer steps with CUDA events while the token batches already sit
on the device; ``e2e`` times K further steps by wall clock through ``Trainer.train_step`` with every step's batch
copied from pinned host memory and its loss read back.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PRESETS = {
    # name: (d_model, n_layers, n_heads, ff_proj width, micro-batch per GPU, official global batch, flavour)
    "olmo2-7b": dict(d_model=4096, n_layers=32, n_heads=32, mlp_hidden_size=22016, microbatch=2, global_batch=1024, flavour="olmo2"),
    "olmo2-1b": dict(d_model=2048, n_layers=16, n_heads=16, mlp_hidden_size=16384, microbatch=8, global_batch=512, flavour="olmo2"),
    "olmo2-13b": dict(d_model=5120, n_layers=40, n_heads=40, mlp_hidden_size=27648, microbatch=1, global_batch=1024, flavour="olmo2"),
    "olmo1-7b": dict(d_model=4096, n_layers=32, n_heads=32, mlp_hidden_size=22016, microbatch=2, global_batch=1024, flavour="olmo1"),
    "tiny": dict(d_model=256, n_layers=4, n_heads=2, mlp_hidden_size=2048, microbatch=2, global_batch=16, flavour="olmo2"),
}


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", choices=sorted(PRESETS), default="olmo2-7b")
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--device-batch", type=int, default=None,
                   help="sequences per GPU per optimizer step (default: 32; the official global batch / 8 is 128 for the 7B preset)")
    p.add_argument("--activation-checkpointing", default=None)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--sharding", default="FULL_SHARD", choices=["FULL_SHARD", "SHARD_GRAD_OP", "HYBRID_SHARD", "NO_SHARD"],
                   help="sharding strategy of the flat-shard engine (HYBRID_SHARD: --replicas groups)")
    p.add_argument("--replicas", type=int, default=None, help="model replicas for HYBRID_SHARD (default: 2)")
    p.add_argument("--checkpoint-timing", action="store_true",
                   help="after the timed steps also time a sharded checkpoint save, its restore and the offline unshard")
    p.add_argument("--n-layers", type=int, default=None, help="profiling aid: fewer blocks than the preset (the result is then marked reduced)")
    p.add_argument("--schedule", choices=["auto", "resident", "sharded"], default="auto",
                   help="FULL_SHARD execution schedule of the flat-shard engine: 'resident' keeps every unit gathered between uses "
                        "(one gather and one reduce-scatter per unit and optimizer step), 'sharded' streams the block units "
                        "(gather in forward and backward, reduce-scatter every micro-batch), 'auto' takes resident while it fits")
    p.add_argument("--no-check", action="store_true", help="skip the comparison of the peer-memory collectives with NCCL before the timed region")
    return p.parse_args()


def make_train_config(args, world: int):
    from olmo_b200.config import (
        ActivationCheckpointingStrategy, DistributedStrategy, FSDPConfig, FSDPPrecision, FSDPWrapStrategy, InitFnType,
        LayerNormType, ModelConfig, OptimizerConfig, OptimizerType, SchedulerConfig, SchedulerType, SchedulerUnits,
        ShardingStrategy, SpeedMonitorConfig, TrainConfig,
    )

    ps = PRESETS[args.model]
    olmo2 = ps["flavour"] == "olmo2"
    model = ModelConfig(
        d_model=ps["d_model"], n_heads=ps["n_heads"], n_layers=args.n_layers or ps["n_layers"], mlp_hidden_size=ps["mlp_hidden_size"],
        weight_tying=False, alibi=False, rope=True, rope_theta=500000 if olmo2 else 10000, flash_attention=True,
        attention_dropout=0.0, include_bias=False, layer_norm_type=LayerNormType.rms if olmo2 else LayerNormType.default,
        layer_norm_with_affine=olmo2, layer_norm_eps=1e-6 if olmo2 else 1e-5, bias_for_layer_norm=False,
        attention_layer_norm=olmo2, attention_layer_norm_with_affine=olmo2, norm_after=olmo2, residual_dropout=0.0,
        embedding_dropout=0.0, max_sequence_length=args.seq_len, vocab_size=100278 if olmo2 else 50280,
        embedding_size=100352 if olmo2 else 50304, eos_token_id=100257 if olmo2 else 50279, pad_token_id=100277 if olmo2 else 1,
        init_device="meta", init_fn=InitFnType.normal if olmo2 else InitFnType.mitchell, init_std=0.02,
        init_cutoff_factor=3 if olmo2 else None, clip_qkv=None if olmo2 else 8.0,
    )
    device_batch = args.device_batch or max(ps["microbatch"], min(32, ps["global_batch"] // 8))
    cfg = TrainConfig(
        run_name=f"bench-{args.model}", model=model,
        optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=3e-4, weight_decay=0.1, eps=1e-8, betas=(0.9, 0.95),
                                  decay_norm_and_bias=True, decay_embeddings=False),
        scheduler=SchedulerConfig(name=SchedulerType.cosine_with_warmup, units=SchedulerUnits.tokens, t_warmup=8388608000, t_max=5e12,
                                  alpha_f=0.1, warmup_min_lr=0.0),
        global_train_batch_size=device_batch * world, device_train_microbatch_size=ps["microbatch"], precision="amp_bf16",
        distributed_strategy=DistributedStrategy.fsdp,
        fsdp=FSDPConfig(sharding_strategy=ShardingStrategy[args.sharding], wrapping_strategy=FSDPWrapStrategy.by_block_and_size,
                        precision=FSDPPrecision.mixed,
                        hybrid_sharding_num_model_replicas=(args.replicas or 2) if args.sharding == "HYBRID_SHARD" else None),
        max_grad_norm=1.0, softmax_auxiliary_loss=True, auxiliary_loss_multiplier=1e-5, fused_loss=True,
        save_folder=tempfile.mkdtemp(prefix="olmo_b200_bench_"), save_overwrite=True, save_data_indices=False,
        max_duration=10**9, console_log_interval=10**9, speed_monitor=SpeedMonitorConfig(window_size=1),
        activation_checkpointing=None if args.activation_checkpointing in (None, "none") else ActivationCheckpointingStrategy(args.activation_checkpointing),
    )
    return cfg, device_batch


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU with nvidia-smi while the timed region runs."""

    FIELDS = "timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int, interval_ms: int = 200):
        self.index, self.proc, self.path, self.interval_ms = index, None, None, interval_ms
        self.samples = []  # (seconds since the epoch, SM MHz, watts) of every sample, filled by stop()

    def start(self) -> None:
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            pass
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            try:
                stamp = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                self.samples.append((stamp, sm[-1], float(parts[3])))
            except ValueError:
                pass
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons), "samples": len(sm)}


def bench_config(args, ps: dict, device_batch: int, world: int, grad_accum: int) -> dict:
    """The ``config`` entry of the JSON line.  Both arms call this, so the two lines carry the same keys and values."""
    return {
        "model": args.model, "global_batch": device_batch * world, "seq_len": args.seq_len, "micro_batch": ps["microbatch"],
        "grad_accum": grad_accum,
        "parallelism": f"fsdp {args.sharding.lower()} x{world}" + (f" ({args.replicas or 2} replicas)" if args.sharding == "HYBRID_SHARD" else ""),
        "activation_checkpointing": args.activation_checkpointing or "none",
        "l2": "inputs larger than L2: each step touches >100 GB of parameters, optimizer state and activations",
    }


class PhaseTimer:
    """CUDA events at the phase boundaries of one training step (the engine and the optimizer call ``mark``)."""

    def __init__(self) -> None:
        self.marks = []

    def mark(self, name: str) -> None:
        import torch

        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks.append((name, ev))

    def summary(self, world: int, device) -> dict:
        """Milliseconds per phase, summed over the step, as min / median / max over ranks.  A mark names the phase that
        *starts* there; ``barrier_wait`` is the end-of-step scalar all-reduce, whose duration is the time this rank spent
        waiting for the slowest rank."""
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        names = ["forward", "backward", "grad_sync", "barrier_wait", "clip", "optimizer"]
        acc = {n: 0.0 for n in names}
        for (name, ev), (_, nxt) in zip(self.marks, self.marks[1:]):
            if name in acc:
                acc[name] += ev.elapsed_time(nxt)
        t = torch.tensor([acc[n] for n in names], device=device, dtype=torch.float64)
        if world > 1:
            every = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(every, t)
            m = torch.stack(every)
        else:
            m = t[None]
        return {n: {"min": m[:, i].min().item(), "median": m[:, i].median().item(), "max": m[:, i].max().item()} for i, n in enumerate(names)}


def clocks_by_phase(samples, t0: float, boundaries) -> dict:
    """Median SM clock and power per phase.  ``samples``: (epoch seconds, MHz, watts); ``t0``: epoch seconds at which the
    device started the step; ``boundaries``: (phase name, start offset in ms, end offset in ms) in device time."""
    bins = {}
    for stamp, mhz, watts in samples:
        off = (stamp - t0) * 1e3
        for name, a, b in boundaries:
            if a <= off < b:
                bins.setdefault(name, []).append((mhz, watts))
                break
    return {name: {"sm_mhz": statistics.median(v[0] for v in vals), "power_w": statistics.median(v[1] for v in vals), "samples": len(vals)}
            for name, vals in bins.items()}


def run_ours(args) -> dict:
    import torch
    import torch.distributed as dist

    from olmo_b200 import ops
    from olmo_b200.data import SyntheticTokenDataset
    from olmo_b200.launch import build_trainer, derive_batch_sizes
    from olmo_b200.ops import kernels

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"

    os.environ["OLMO_B200_SCHEDULE"] = args.schedule
    cfg, device_batch = make_train_config(args, world)
    if world > 1:  # one save folder for the whole job (every rank made its own temporary directory)
        shared = [cfg.save_folder]
        dist.broadcast_object_list(shared, src=0)
        cfg.save_folder = shared[0]
        os.environ.setdefault("OLMO_SHARED_FS", "1")
    derive_batch_sizes(cfg, world)
    ps = PRESETS[args.model]
    trainer = build_trainer(cfg, device=device, train_loader=_dummy_loader(), with_evaluators=False)
    engine = trainer.dist_model.engine
    model = trainer.model
    flops_per_token = model.num_fwd_flops + model.num_bck_flops
    n_params = model.num_params()

    data = SyntheticTokenDataset(1 << 20, args.seq_len, cfg.model.vocab_size, cfg.model.eos_token_id, seed=cfg.seed)
    total_steps = args.warmup + 2 * args.steps + 1
    host_batches = [data.batch((s * world + rank) * device_batch, device_batch, pin=True) for s in range(min(total_steps, 4))]

    def step(i: int, from_host: bool) -> float:
        ids = host_batches[i % len(host_batches)]
        batch = {"input_ids": ids if from_host else dev_batches[i % len(dev_batches)]}
        trainer.global_step += 1
        trainer.global_train_tokens_seen += device_batch * world * args.seq_len
        return trainer.train_step(batch, reduce_global_loss=False)["train/CrossEntropyLoss"]

    dev_batches = [b.to(device) for b in host_batches]
    torch.cuda.synchronize()
    loss = float("nan")
    for i in range(args.warmup):
        loss = step(i, False)

    def barrier() -> None:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- the peer-memory collectives of the last warm-up step against NCCL on the same buffers
    multi_gpu_check = None
    if world > 1 and not args.no_check and getattr(engine, "comm", None) is not None:
        multi_gpu_check = engine.verify_collectives_against_nccl()

    # ---- device-timed region
    sampler = ClockSampler(local_rank)
    barrier()
    sampler.start()
    launches0 = kernels.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        loss = step(args.warmup + i, False)
    ev1.record()
    barrier()
    clocks = sampler.stop()
    launches = kernels.launch_count() - launches0
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = t.item() / args.steps

    # ---- end-to-end region (pinned host batch -> device every step, loss read back every step)
    e2e = None
    if not args.no_e2e:
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            loss = step(args.warmup + args.steps + i, True)
        barrier()
        wall = torch.tensor([time.perf_counter() - t0], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(wall, op=dist.ReduceOp.MAX)
        e2e_tokens = device_batch * world * args.seq_len * args.steps
        e2e = {
            "value": e2e_tokens / wall.item(), "unit": "tokens/s",
            "h2d_bytes_per_step": device_batch * args.seq_len * 8, "d2h_bytes_per_step": 16,
            "ms_per_step": wall.item() * 1e3 / args.steps,
        }

    # ---- one more step with per-phase CUDA events on every rank (not part of either timed region)
    phases = phase_clocks = None
    if engine.fused:
        engine.phase_timer = PhaseTimer()
        # a short, odd interval: the 200 ms of the timed region is close to a multiple of a micro-batch's duration for some
        # model sizes, and then every sample would fall into the same phase
        phase_sampler = ClockSampler(local_rank, interval_ms=37)
        phase_sampler.start()
        time.sleep(0.5)  # the sampler needs a moment to produce its first line
        barrier()
        t_host0 = time.time()  # the device is idle here, so the event below is recorded at this moment
        ev_p0 = torch.cuda.Event(enable_timing=True)
        ev_p0.record()
        step(args.warmup + 2 * args.steps, False)
        barrier()
        phase_sampler.stop()
        marks = engine.phase_timer.marks
        bounds = [(name, ev_p0.elapsed_time(ev), ev_p0.elapsed_time(nxt)) for (name, ev), (_, nxt) in zip(marks, marks[1:])]
        phase_clocks = clocks_by_phase(phase_sampler.samples, t_host0, bounds)
        phases = engine.phase_timer.summary(world, device)
        engine.phase_timer = None

    checkpoint = None
    if args.checkpoint_timing:
        checkpoint = time_checkpoint_cycle(trainer, cfg, rank, world, barrier)

    tokens_per_step = device_batch * world * args.seq_len
    value = tokens_per_step / (ms_per_step / 1e3)
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    per_gpu = value / world
    schedule = getattr(engine, "schedule", "resident") if world > 1 else "single device"
    sm_mhz = clocks.get("sm_mhz")
    result = {
        "metric": f"tokens_per_second ({'OLMo-2' if ps['flavour'] == 'olmo2' else 'OLMo-1'} training, whole job; FSDP {args.sharding}, {schedule} schedule, device-timed, max over ranks)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic seeded uniform tokens with EOS boundaries; random-init weights",
        "impl": "ours",
        "tokens_per_second_per_gpu": per_gpu,
        "mfu_nominal_2250tf": per_gpu * flops_per_token / 2.25e15,
        "mfu_of_measured_sustained": (per_gpu * flops_per_token / (peaks["bf16_tflops_sustained"] * 1e12)) if peaks.get("bf16_tflops_sustained") else None,
        "flops_per_token": flops_per_token, "params": n_params, "final_loss": loss,
        # the same keys, with the same values, as the reference arm prints for the same command line
        "config": bench_config(args, ps, device_batch, world, cfg.device_train_grad_accum),
        "schedule": schedule,
        "schedule_note": {
            "resident": "every unit stays gathered between uses: one gather and one reduce-scatter per unit and optimizer step (what SHARD_GRAD_OP asks for; FULL_SHARD gets it while it fits)",
            "sharded": "block units are streamed: gathered in forward and again in backward, gradients reduce-scattered every micro-batch, all from inside the block GEMM launches",
        }.get(schedule, "one device: nothing to gather or reduce"),
        "implementation": {
            "engine": "flat-shard engine, peer-memory collectives" if getattr(engine, "comm", None) is not None else ("flat-shard engine" + (", NCCL collectives" if world > 1 else "")),
            "official_global_batch_at_8_gpus": ps["global_batch"], "sequences_per_gpu_per_step": device_batch,
            "optimizer": "adamw fp32 master, clip 1.0, z-loss on", "fused_path": bool(engine.fused),
            "recomputable_activations": "kept" if getattr(engine, "keep_recomputable", False) else "recomputed in backward",
            "reduced_model": f"REDUCED to {args.n_layers} layers (profiling only)" if args.n_layers else None,
        },
        "ms_per_step_x_sm_ghz": (ms_per_step * sm_mhz / 1e3) if sm_mhz else None,
        "phases_ms": phases, "clocks_by_phase_rank0": phase_clocks, "multi_gpu_check": multi_gpu_check,
        "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "checkpoint": checkpoint,
        "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9,
        # the caching allocator's peak does not see peer-memory (symmetric) buffers; this is the device's own count
        "device_mem_in_use_gb": (lambda free_total: (free_total[1] - free_total[0]) / 1e9)(torch.cuda.mem_get_info()),
    }
    if world > 1:
        dist.destroy_process_group()
    return result if rank == 0 else {}


def time_checkpoint_cycle(trainer, cfg, rank: int, world: int, barrier) -> dict:
    """Wall-clock seconds (max over ranks) of a sharded save, a restore of it, and the offline unshard on rank 0."""
    import torch
    import torch.distributed as dist

    from olmo_b200.checkpoint import build_sharded_checkpointer

    def timed(fn) -> float:
        barrier()
        t0 = time.perf_counter()
        out = fn()
        barrier()
        t = torch.tensor([time.perf_counter() - t0], device=trainer.device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        timed.last = out
        return t.item()

    save_s = timed(trainer.save_checkpoint)
    path = timed.last[0]
    restore_s = timed(lambda: trainer.restore_checkpoint(path))
    unshard_s = None
    if rank == 0:
        t0 = time.perf_counter()
        build_sharded_checkpointer(cfg).unshard_checkpoint(path, load_optimizer_state=True, load_trainer_state=True)
        unshard_s = time.perf_counter() - t0
    barrier()
    size = sum(f.stat().st_size for f in Path(path).rglob("*") if f.is_file()) if rank == 0 else 0
    return {"sharded_save_s": save_s, "restore_s": restore_s, "unshard_s": unshard_s, "bytes_on_disk": size, "path": str(path)}


def _dummy_loader():
    from torch.utils.data import DataLoader

    from olmo_b200.data import IterableDataset

    return DataLoader(IterableDataset([[0]], 1, world_size=1, rank=0, fs_local_rank=0, num_threads=0), batch_size=1)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        from baseline.ref_bench import run_reference

        out = run_reference(args, PRESETS)
    else:
        out = run_ours(args)
    if out:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
