"""In-loop evaluation builders (reference: ``olmo/eval/__init__.py:24-114``)."""
from __future__ import annotations

from typing import Dict, List, Union

import torch
from torch.utils.data import DataLoader, DistributedSampler

from ..config import EvaluatorConfig, EvaluatorType, TrainConfig
from ..exceptions import OLMoConfigurationError
from ..torch_util import get_global_rank, get_world_size
from .evaluator import Evaluator
from .metrics import ICLMetric, MeanMetric, Metric

__all__ = ["Evaluator", "ICLMetric", "MeanMetric", "Metric", "build_downstream_evaluator", "build_evaluator", "build_evaluators"]


def build_downstream_evaluator(train_config: TrainConfig, eval_cfg: EvaluatorConfig, tokenizer, device: torch.device, is_unit_test: bool = False) -> Evaluator:
    from .downstream import label_to_task_map

    task_kwargs = {}
    task_class = label_to_task_map[eval_cfg.label]
    if isinstance(task_class, tuple):
        task_class, task_kwargs = task_class
    ds_eval_dataset = task_class(tokenizer=tokenizer, **task_kwargs)
    data_config = eval_cfg.data
    if is_unit_test:
        ds_eval_sampler = None
    else:
        ds_eval_sampler = DistributedSampler(
            ds_eval_dataset, drop_last=data_config.drop_last, shuffle=False, num_replicas=get_world_size(), rank=get_global_rank(), seed=train_config.seed,
        )
    workers = data_config.num_workers
    ds_eval_dataloader = DataLoader(
        ds_eval_dataset,
        batch_size=eval_cfg.device_eval_batch_size or train_config.device_eval_batch_size,
        collate_fn=ds_eval_dataset.collate_fn,
        num_workers=workers,
        sampler=ds_eval_sampler,
        pin_memory=data_config.pin_memory,
        prefetch_factor=None if workers == 0 else data_config.prefetch_factor,
        persistent_workers=False if workers == 0 else data_config.persistent_workers,
        timeout=data_config.timeout,
    )
    metric = ICLMetric(metric_type=ds_eval_dataset.metric_type)
    return Evaluator(label=eval_cfg.label, type=eval_cfg.type, eval_loader=ds_eval_dataloader, eval_metric=metric.to(device), subset_num_batches=eval_cfg.subset_num_batches)


def build_evaluator(train_config: TrainConfig, eval_config: EvaluatorConfig, tokenizer, device: torch.device) -> Evaluator:
    from ..data import build_eval_dataloader

    if eval_config.type == EvaluatorType.downstream:
        return build_downstream_evaluator(train_config, eval_config, tokenizer, device)
    if eval_config.type == EvaluatorType.lm:
        loader = build_eval_dataloader(train_config, eval_config.data, eval_config.device_eval_batch_size or train_config.device_eval_batch_size)

        def make_metric() -> MeanMetric:
            return MeanMetric().to(device)

        eval_metric: Union[Metric, Dict[str, Metric]]
        if eval_config.data.paths:
            eval_metric = make_metric()
        elif eval_config.data.datasets:
            eval_metric = {label: make_metric() for label in eval_config.data.datasets.keys()}
        else:
            raise OLMoConfigurationError("One of DataConfig.paths or DataConfig.datasets is required")
        return Evaluator(label=eval_config.label, type=eval_config.type, eval_loader=loader, eval_metric=eval_metric, subset_num_batches=eval_config.subset_num_batches)
    raise ValueError(f"Unexpected evaluator type '{eval_config.type}'")


def build_evaluators(cfg: TrainConfig, device: torch.device) -> List[Evaluator]:
    if not cfg.evaluators:
        return []
    tokenizer = None
    if any(e.type == EvaluatorType.downstream for e in cfg.evaluators):
        # only in-context tasks render text; perplexity evaluators read token files and need no vocabulary
        from ..tokenizer import Tokenizer

        tokenizer = Tokenizer.from_train_config(cfg)
    return [build_evaluator(cfg, eval_cfg, tokenizer, device) for eval_cfg in cfg.evaluators]
