"""
One evaluation stream of the training loop: a loader, its metric state, and the names its results are logged under.

The public face is the dataclass the reference defines in ``olmo/eval/evaluator.py:14-85`` (fields ``label``, ``type``,
``eval_loader``, ``eval_metric``, ``subset_num_batches``; methods ``reset_metrics`` / ``update_metrics`` /
``compute_metrics``), and the logged keys are the same: ``eval/{label}/CrossEntropyLoss`` and ``…/Perplexity`` for token
files, ``eval/downstream/{label}_{metric}`` for in-context tasks (``eval/downstream_{metric}/…`` for the two loss-like
metrics).  How a batch updates the state and how the state becomes numbers is decided once, by a scorer picked from
the evaluator type.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Optional, Union

import torch
from torch.utils.data import DataLoader

from ..config import EvaluatorType
from .metrics import ICLMetric, MeanMetric, Metric

__all__ = ["Evaluator"]

_LOSS_LIKE = ("ce_loss", "bpb")  # in-context metrics that are logged under their own prefix


class _TaskScorer:
    """An in-context task: the metric consumes the batch and the logits; one number comes out."""

    def __init__(self, label: str, metric: ICLMetric):
        self.metrics = [metric]
        kind = metric.metric_type
        prefix = f"eval/downstream_{kind}" if kind in _LOSS_LIKE else "eval/downstream"
        self.key = f"{prefix}/{label}_{kind}"

    def update(self, batch: Dict[str, Any], ce_loss: torch.Tensor, logits: torch.Tensor) -> None:
        self.metrics[0].update(batch, logits)

    def results(self) -> Dict[str, float]:
        return {self.key: self.metrics[0].compute().item()}


class _PerplexityScorer:
    """Token files: a running mean of the per-instance loss, one per label when instances carry labels."""

    def __init__(self, label: str, metric: Union[MeanMetric, Dict[str, MeanMetric]]):
        self.by_label = metric if isinstance(metric, dict) else None
        self.single = None if isinstance(metric, dict) else (label, metric)
        self.metrics = list(metric.values()) if isinstance(metric, dict) else [metric]

    def update(self, batch: Dict[str, Any], ce_loss: torch.Tensor, logits: torch.Tensor) -> None:
        for meta, loss in zip(batch["metadata"], ce_loss):
            (self.by_label[meta["label"]] if self.by_label is not None else self.single[1]).update(loss)

    def results(self) -> Dict[str, float]:
        named = sorted(self.by_label.items()) if self.by_label is not None else [self.single]
        out: Dict[str, float] = {}
        for label, metric in named:
            mean = metric.compute()
            if torch.isnan(mean):  # this label saw no instance in the (possibly truncated) pass
                continue
            out[f"eval/{label}/CrossEntropyLoss"] = mean.item()
            out[f"eval/{label}/Perplexity"] = mean.exp().item()
        return out


@dataclass
class Evaluator:
    label: str
    type: EvaluatorType
    eval_loader: DataLoader
    eval_metric: Union[Metric, Dict[str, Metric]]
    subset_num_batches: Optional[int] = None
    _scorer: Any = field(init=False, repr=False, compare=False, default=None)

    def __post_init__(self) -> None:
        if self.type == EvaluatorType.downstream:
            assert isinstance(self.eval_metric, ICLMetric)
            self._scorer = _TaskScorer(self.label, self.eval_metric)
        elif self.type == EvaluatorType.lm:
            self._scorer = _PerplexityScorer(self.label, self.eval_metric)  # type: ignore[arg-type]
        else:
            raise ValueError(f"Unexpected evaluator type '{self.type}'")

    def reset_metrics(self) -> None:
        for metric in self._scorer.metrics:
            metric.reset()

    def update_metrics(self, batch: Dict[str, Any], ce_loss: torch.Tensor, logits: torch.Tensor) -> None:
        self._scorer.update(batch, ce_loss, logits)

    def compute_metrics(self) -> Dict[str, float]:
        return self._scorer.results()
