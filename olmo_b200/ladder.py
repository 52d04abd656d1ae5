"""
Scaling-ladder config synthesis: given a model size rung ("150M" … "7B"), a training length ("2xC" = twice
Chinchilla-optimal, or "10B" tokens) and a data mix, derive the whole :class:`TrainConfig` — batch size and peak learning
rate follow the power laws of the reference's ``scripts/ladder.py:152-170``:

* global batch  = 160 · (N / 108e6)^(2/3) sequences of 2048 tokens, rounded to a multiple of 32;
* peak LR       = 0.0047 · (N / 108e6)^(-1/3);
* warm-up       = N / (batch · seq_len) steps (one token per parameter), cosine decay to 1 % of peak.

B200 specifics: a rung up to 1B trains with replicated parameters (DDP) and the 7B rung with the flat-shard engine, as
in the reference, but micro-batch sizes are chosen for 180 GB parts.
"""
from __future__ import annotations

import re
from copy import deepcopy
from typing import Any, Dict, List, Optional, Set, Tuple

from .config import (
    DataConfig, DDPConfig, DistributedStrategy, EvaluatorConfig, EvaluatorType, FSDPConfig, FSDPPrecision, FSDPWrapStrategy,
    InstanceFilterConfig, ModelConfig, OptimizerConfig, OptimizerType, SchedulerConfig, SchedulerType, ShardedCheckpointerType,
    ShardingStrategy, SpeedMonitorConfig, TokenizerConfig, TrainConfig, WandbConfig,
)
from .recipes import DEFAULT_EVALUATORS, _TINY_BASE

__all__ = ["RUNGS", "parse_size", "parse_length", "batch_size_for", "learning_rate_for", "ladder_config", "node_counts", "size_for_model"]

_LADDER_BASE: Dict[str, Any] = {**_TINY_BASE, "max_sequence_length": 2048, "eos_token_id": 50279, "init_device": "cuda"}
RUNGS: Dict[str, Dict[str, Any]] = {
    "150M": dict(d_model=768, n_heads=12, n_layers=12),
    "300M": dict(d_model=1024, n_heads=16, n_layers=16),
    "750M": dict(d_model=1536, n_heads=16, n_layers=16),
    "1B": dict(d_model=2048, n_heads=16, n_layers=16),
    "7B": dict(d_model=4096, n_heads=32, n_layers=32, mlp_ratio=0, mlp_hidden_size=22016, init_device="meta"),
}
#: sequences per GPU per micro-batch on a 180 GB part (activations of one micro-batch stay below ~40 GB)
MICROBATCH = {"150M": 32, "300M": 16, "750M": 8, "1B": 8, "7B": 4}
_PPL_SETS = [
    "c4_en", "dolma_books", "dolma_common-crawl", "dolma_pes2o", "dolma_reddit", "dolma_stack", "dolma_wiki", "ice", "m2d2_s2orc",
    "pile", "wikitext_103",
]
_NUM_UNIT = re.compile(r"^([0-9]+)([a-zA-Z]+)$")
_SCALE = {"K": 10**3, "M": 10**6, "B": 10**9, "T": 10**12}


def parse_size(size: str) -> int:
    m = _NUM_UNIT.match(size.strip().upper())
    if m is None or m.group(2) not in ("K", "M", "B"):
        raise ValueError(f"Could not parse model size '{size}'")
    return int(m.group(1)) * _SCALE[m.group(2)]


def parse_length(length: str, model_size: int) -> int:
    m = _NUM_UNIT.match(length.strip().upper())
    if m is None:
        raise ValueError(f"Could not parse length '{length}'")
    n, unit = int(m.group(1)), m.group(2)
    if unit in ("C", "XC"):
        return n * 20 * model_size  # multiples of the Chinchilla-optimal 20 tokens per parameter
    if unit in _SCALE:
        return n * _SCALE[unit]
    raise ValueError(f"Could not parse length '{length}'")


def batch_size_for(model_size: int) -> int:
    return round(160 * (model_size / 108_000_000) ** (2 / 3) / 32) * 32


def learning_rate_for(model_size: int) -> float:
    return 0.0047 * (model_size / 108_000_000) ** (-1 / 3)


def model_config_for(rung: str) -> ModelConfig:
    from .utils import structured as S

    try:
        return S.build(ModelConfig, {**_LADDER_BASE, **RUNGS[rung]})
    except KeyError:
        raise KeyError(f"unknown ladder rung '{rung}'; known: {sorted(RUNGS)}") from None


def ladder_config(
    model: str, length: str = "2xC", name: str = "ladder", data: Optional[str] = None, *, read_location: str = "/data",
    remote_save_folder: Optional[str] = None, load_path: Optional[str] = None, wandb: bool = False, save_overwrite: bool = False,
    eval_on_load: bool = False,
) -> TrainConfig:
    rung = model.strip().upper()
    model_cfg = model_config_for(rung)
    n = parse_size(rung)
    tokens = parse_length(length, n)
    batch = batch_size_for(n)
    micro = MICROBATCH.get(rung, 4)
    while batch % micro:
        micro //= 2
    run_name = f"{name}-{rung}-{length}"
    assert "/" not in run_name
    root = read_location.rstrip("/")
    save_interval = {"1B": 2500, "7B": 1000}.get(rung, 5000)
    paths: Optional[List[str]] = None
    if data is not None:
        from .data.named_data_mixes import resolve_mix

        paths = resolve_mix(data, root)
    evaluators = [
        EvaluatorConfig(
            label="all-small-ppl-validation",
            data=DataConfig(drop_last=True, datasets={
                f"{s}-validation": [f"{root}/eval-data/perplexity/v3_small_gptneox20b/{s}/val/part-0-00000.npy"] for s in _PPL_SETS
            }),
        )
    ] + [EvaluatorConfig(label=label, type=EvaluatorType.downstream) for label in DEFAULT_EVALUATORS]
    return TrainConfig(
        run_name=run_name, seed=6198, wandb=WandbConfig(name=run_name, group=run_name, project="olmo-ladder") if wandb else None,
        model=model_cfg, ddp=DDPConfig(),
        fsdp=FSDPConfig(sharding_strategy=ShardingStrategy.SHARD_GRAD_OP, wrapping_strategy=FSDPWrapStrategy.by_block_and_size, precision=FSDPPrecision.mixed),
        optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=learning_rate_for(n), weight_decay=0.05, eps=1e-8,
                                  decay_norm_and_bias=True, decay_embeddings=True, betas=(0.9, 0.95), metrics_log_interval=10),
        scheduler=SchedulerConfig(name=SchedulerType.cosine_with_warmup, alpha_f=0.01, warmup_min_lr=0.0,
                                  t_warmup=round(n / (batch * model_cfg.max_sequence_length))),
        max_duration=f"{tokens}T", global_train_batch_size=batch,
        tokenizer=TokenizerConfig(identifier="tokenizers/allenai_gpt-neox-olmo-dolma-v1_5.json"),
        save_folder=f"runs/{run_name}", remote_save_folder=remote_save_folder, save_overwrite=save_overwrite,
        save_interval_unsharded=save_interval, save_num_unsharded_checkpoints_to_keep=-1, save_interval=None, load_path=load_path,
        eval_on_load=eval_on_load, sharded_checkpointer=ShardedCheckpointerType.olmo_core, device_train_microbatch_size=micro,
        precision="amp_bf16", distributed_strategy=DistributedStrategy.fsdp if rung == "7B" else DistributedStrategy.ddp,
        fused_loss=True, gen1_gc_interval=2, max_grad_norm=1.0, speed_monitor=SpeedMonitorConfig(window_size=1),
        eval_interval=save_interval, device_eval_batch_size=micro, evaluators=evaluators,
        data=DataConfig(num_workers=8, drop_last=True, pin_memory=True, prefetch_factor=8, persistent_workers=True,
                        instance_filter=InstanceFilterConfig(), paths=paths),
    )


def _factors(n: int) -> Set[int]:
    return {f for i in range(1, int(n**0.5) + 1) if n % i == 0 for f in (i, n // i)}


def node_counts(cfg: TrainConfig, gpus_per_node: int = 8) -> List[int]:
    """Node counts (descending) on which the global batch splits into whole micro-batches per GPU."""
    if cfg.global_train_batch_size % cfg.device_train_microbatch_size != 0:
        raise ValueError("Microbatchsize must divide global batch size evenly.")
    gpus = cfg.global_train_batch_size // cfg.device_train_microbatch_size
    if gpus % gpus_per_node != 0:
        raise ValueError(
            f"With {cfg.global_train_batch_size} bz, {cfg.device_train_microbatch_size} mbz, and {gpus_per_node} GPUs per node, "
            "it's impossible to allocate whole nodes."
        )
    return sorted(_factors(gpus // gpus_per_node), reverse=True)


def size_for_model(model_config) -> Tuple[int, int]:
    """``(parameters, non-embedding parameters)`` computed from one instantiated block, so that 7B needs no 7B allocation."""
    from .models.olmo import OLMo

    if isinstance(model_config, str):
        model_config = model_config_for(model_config.strip().upper())
    cfg = deepcopy(model_config)
    cfg.init_device = "meta"
    layers, cfg.n_layers = cfg.n_layers, 1
    one = OLMo(cfg, init_params=False)
    per_block = sum(p.numel() for p in one.transformer.blocks[0].parameters())
    extra = per_block * (layers - 1)
    return one.num_params() + extra, one.num_params(include_embedding=False) + extra


# ------------------------------------------------------------------------------------------- analysis


_RUN_NAME = re.compile(r"^(?P<name>.+)-(?P<size>\d+[KMB])-(?P<length>\d+x?C|\d+[KMBT])$", re.IGNORECASE)


def parse_run_name(run: str) -> Tuple[str, str, str]:
    """``baseline-300M-5xC`` -> ``("baseline", "300M", "5xC")`` (the naming scheme of ``scripts/ladder.py train --name``)."""
    m = _RUN_NAME.match(run.strip())
    if m is None:
        raise ValueError(f"'{run}' is not a ladder run name (<name>-<size>-<length>)")
    return m.group("name"), m.group("size").upper(), m.group("length")


def power_law(x, a: float, b: float, c: float):
    """``a * x**b + c`` with ``b <= 0``: the irreducible loss ``c`` plus a term that shrinks with scale."""
    return a * x**b + c


def fit_power_law(x: List[float], y: List[float]) -> Tuple[float, float, float]:
    """Least-squares ``(a, b, c)`` of :func:`power_law` under ``a >= 0``, ``b <= 0``, ``c >= 0`` (what the reference's
    ``scripts/ladder.ipynb`` fits to ladder results).  ``x`` is rescaled internally so that parameter counts of 1e8–1e10
    do not wreck the conditioning."""
    import numpy as np
    from scipy.optimize import curve_fit

    xs, ys = np.asarray(x, dtype=np.float64), np.asarray(y, dtype=np.float64)
    if len(xs) < 3:
        raise ValueError("a three-parameter power law needs at least three points")
    scale = float(xs.min())
    guess = (max(ys.max() - ys.min(), 1e-3), -0.3, max(ys.min() * 0.8, 0.0))
    (a, b, c), _ = curve_fit(power_law, xs / scale, ys, p0=guess, bounds=([0, -np.inf, 0], [np.inf, 0, np.inf]), maxfev=20000)
    return float(a * scale ** (-b)), float(b), float(c)


def ladder_fit(results: Dict[str, float], by: str = "size", hold_out: int = 1) -> Dict[str, Any]:
    """Fit loss against model size (non-embedding parameters) or against training length (tokens) over the runs in
    ``results`` (run name -> loss), keeping the ``hold_out`` largest ones aside, and report how well they are predicted."""
    points = []
    for run, loss in results.items():
        _, size, length = parse_run_name(run)
        _, non_embedding = size_for_model(size)
        x = non_embedding if by == "size" else parse_length(length, non_embedding)
        points.append((float(x), float(loss), run))
    points.sort()
    train = points[: len(points) - hold_out] if hold_out else points
    a, b, c = fit_power_law([p[0] for p in train], [p[1] for p in train])
    rows = [{"run": run, "x": x, "loss": loss, "predicted": power_law(x, a, b, c), "held_out": i >= len(train)}
            for i, (x, loss, run) in enumerate(points)]
    return {"a": a, "b": b, "c": c, "by": by, "points": rows}
