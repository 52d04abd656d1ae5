"""Builders for the evaluators that run inside the training loop (public functions of ``olmo/eval/__init__.py:24-114``)."""
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


def _eval_batch_size(train_config: TrainConfig, eval_cfg: EvaluatorConfig) -> int:
    return eval_cfg.device_eval_batch_size or train_config.device_eval_batch_size


def _as_evaluator(eval_cfg: EvaluatorConfig, loader: DataLoader, metric: Union[Metric, Dict[str, Metric]]) -> Evaluator:
    return Evaluator(label=eval_cfg.label, type=eval_cfg.type, eval_loader=loader, eval_metric=metric, subset_num_batches=eval_cfg.subset_num_batches)


def build_downstream_evaluator(train_config: TrainConfig, eval_cfg: EvaluatorConfig, tokenizer, device: torch.device, is_unit_test: bool = False) -> Evaluator:
    """An in-context task evaluator: the task named by the evaluator's label, strided over the ranks in file order, scored
    with the task's own metric (reference: ``olmo/eval/__init__.py:24-68``)."""
    from ..data import _loader_options
    from .downstream import label_to_task_map

    entry = label_to_task_map[eval_cfg.label]
    task_class, task_kwargs = entry if isinstance(entry, tuple) else (entry, {})
    task = task_class(tokenizer=tokenizer, **task_kwargs)
    sampler = None
    if not is_unit_test:  # unit tests run without a process group
        sampler = DistributedSampler(task, drop_last=eval_cfg.data.drop_last, shuffle=False, num_replicas=get_world_size(),
                                     rank=get_global_rank(), seed=train_config.seed)
    loader = DataLoader(task, batch_size=_eval_batch_size(train_config, eval_cfg), collate_fn=task.collate_fn, sampler=sampler,
                        **_loader_options(eval_cfg.data))
    return _as_evaluator(eval_cfg, loader, ICLMetric(metric_type=task.metric_type).to(device))


def _perplexity_evaluator(train_config: TrainConfig, eval_cfg: EvaluatorConfig, device: torch.device) -> Evaluator:
    """Cross-entropy over token files: one running mean, or one per label when the data section has labelled groups."""
    from ..data import build_eval_dataloader

    data = eval_cfg.data
    if not data.paths and not data.datasets:
        raise OLMoConfigurationError("One of DataConfig.paths or DataConfig.datasets is required")
    loader = build_eval_dataloader(train_config, data, _eval_batch_size(train_config, eval_cfg))
    metric: Union[Metric, Dict[str, Metric]]
    metric = MeanMetric().to(device) if data.paths else {label: MeanMetric().to(device) for label in data.datasets}
    return _as_evaluator(eval_cfg, loader, metric)


def build_evaluator(train_config: TrainConfig, eval_config: EvaluatorConfig, tokenizer, device: torch.device) -> Evaluator:
    """Dispatch on the evaluator type (reference: ``olmo/eval/__init__.py:71-106``)."""
    if eval_config.type == EvaluatorType.downstream:
        return build_downstream_evaluator(train_config, eval_config, tokenizer, device)
    if eval_config.type == EvaluatorType.lm:
        return _perplexity_evaluator(train_config, eval_config, device)
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
