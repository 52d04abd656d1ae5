"""
Assembly of a training run from a :class:`TrainConfig`: device batch arithmetic, model + engine, optimizer,
scheduler, data loader, evaluators and the :class:`Trainer` (what the reference does inline in
``scripts/train.py:46-378``).  Entry scripts, the benchmark and the tests share this code.
"""
from __future__ import annotations

import logging
from pathlib import Path
from typing import Optional

import torch
from torch.utils.data import DataLoader

from .config import DistributedStrategy, TrainConfig
from .exceptions import OLMoConfigurationError
from .models.olmo import OLMo
from .optim import build_optimizer, build_scheduler
from .parallel.fsdp import ShardedModel, build_sharded_model
from .torch_util import get_global_rank, get_world_size
from .train import Trainer

__all__ = ["derive_batch_sizes", "select_device", "build_model_and_engine", "build_trainer"]

log = logging.getLogger(__name__)


def derive_batch_sizes(cfg: TrainConfig, world_size: Optional[int] = None) -> None:
    """Fill ``device_train_batch_size`` and ``device_train_grad_accum`` and the model's precision field."""
    world = world_size or get_world_size()
    if cfg.global_train_batch_size % world != 0:
        raise OLMoConfigurationError("global_train_batch_size must be divisible by the world size")
    cfg.device_train_batch_size = cfg.global_train_batch_size // world
    cfg.device_train_grad_accum = max(1, cfg.device_train_batch_size // cfg.device_train_microbatch_size)
    cfg.model.precision = cfg.precision
    if cfg.fsdp is not None and cfg.fsdp.wrapping_strategy is not None and cfg.distributed_strategy == DistributedStrategy.ddp:
        log.warning("fsdp.wrapping_strategy is ignored with distributed_strategy=ddp")


def select_device(cfg: TrainConfig) -> torch.device:
    if cfg.distributed_strategy == DistributedStrategy.single or not torch.cuda.is_available():
        if cfg.distributed_strategy == DistributedStrategy.single:
            return cfg.single.get_device()
        return torch.device("cpu")
    return torch.device("cuda", torch.cuda.current_device())


def needs_portable_path(cfg: TrainConfig) -> Optional[str]:
    """Why this run cannot use the fused kernel sequence for its training steps, or ``None``.  The choice between the
    fused and the portable (autograd) path is made once, when the engine is built: a fused engine has no autograd graph
    to fall back on for a single odd batch."""
    mc = cfg.model
    if cfg.module_outputs_save_steps:
        return "module_outputs_save_steps records module outputs through forward hooks"
    data = cfg.data
    if data is not None and getattr(data, "generate_doc_lengths", False):
        if mc.d_model // mc.n_heads > 128:
            return "intra-document masking covers head dimensions up to 128 on the fused path"
    if data is not None and getattr(data, "generate_attention_mask", False):
        return "padded batches (generate_attention_mask) carry an attention mask"
    return None


def build_model_and_engine(cfg: TrainConfig, device: torch.device, **engine_kwargs) -> ShardedModel:
    """Instantiate the model without storage, then let the engine materialise, initialise and shard it."""
    why = needs_portable_path(cfg)
    if why is not None and not engine_kwargs.get("force_portable", False):
        log.info("using the portable (autograd) path: %s", why)
        engine_kwargs["force_portable"] = True
    model_cfg = cfg.model
    prior = model_cfg.init_device
    model_cfg.init_device = "meta"
    try:
        model = OLMo(model_cfg, init_params=False)
    finally:
        model_cfg.init_device = prior
    model.set_activation_checkpointing(cfg.activation_checkpointing)
    return build_sharded_model(model, cfg, device, **engine_kwargs)


def build_trainer(
    cfg: TrainConfig, device: Optional[torch.device] = None, train_loader: Optional[DataLoader] = None, with_evaluators: bool = True,
    **engine_kwargs,
) -> Trainer:
    from .data import build_train_dataloader
    from .eval import build_evaluators

    if cfg.device_train_batch_size is None:
        derive_batch_sizes(cfg)
    device = device or select_device(cfg)
    if train_loader is None:
        train_loader = build_train_dataloader(cfg)
    evaluators = build_evaluators(cfg, device) if with_evaluators else []
    dist_model = build_model_and_engine(cfg, device, **engine_kwargs)
    log.info("Total number of parameters: %s", f"{dist_model.module.num_params():,d}")
    log.info("Number of non-embedding parameters: %s", f"{dist_model.module.num_params(include_embedding=False):,d}")
    optim = build_optimizer(cfg, dist_model)
    scheduler = build_scheduler(cfg)
    indices_file = None
    if cfg.save_data_indices and cfg.save_folder:
        import gzip

        path = Path(cfg.save_folder) / "data-indices" / f"rank{get_global_rank()}.tsv.gz"
        if path.exists() and not cfg.save_overwrite:
            raise OLMoConfigurationError(f"{path} already exists, use --save_overwrite to overwrite")
        path.parent.mkdir(exist_ok=True, parents=True)
        indices_file = gzip.open(path, "wt")
    return Trainer(
        cfg=cfg, epoch=cfg.epoch, model=dist_model.module, dist_model=dist_model, optim=optim, scheduler=scheduler,
        train_loader=train_loader, device=device, evaluators=evaluators, indices_file=indices_file,
    )
