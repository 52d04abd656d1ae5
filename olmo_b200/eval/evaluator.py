"""One evaluation stream: a loader plus its metric(s) (reference: ``olmo/eval/evaluator.py:14-85``)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Optional, Union

import torch
from torch.utils.data import DataLoader

from ..config import EvaluatorType
from .metrics import ICLMetric, MeanMetric, Metric

__all__ = ["Evaluator"]


@dataclass
class Evaluator:
    label: str
    type: EvaluatorType
    eval_loader: DataLoader
    eval_metric: Union[Metric, Dict[str, Metric]]
    subset_num_batches: Optional[int] = None

    def _all_metrics(self) -> Dict[str, Metric]:
        return self.eval_metric if isinstance(self.eval_metric, dict) else {self.label: self.eval_metric}

    def reset_metrics(self) -> None:
        for m in self._all_metrics().values():
            m.reset()

    def compute_metrics(self) -> Dict[str, float]:
        if self.type == EvaluatorType.downstream:
            assert isinstance(self.eval_metric, ICLMetric)
            kind = self.eval_metric.metric_type
            key = f"eval/downstream/{self.label}_{kind}"
            if kind in ("ce_loss", "bpb"):
                key = key.replace("/downstream/", f"/downstream_{kind}/")
            return {key: self.eval_metric.compute().item()}
        if self.type == EvaluatorType.lm:
            out: Dict[str, float] = {}
            for label, metric in sorted(self._all_metrics().items()):
                assert isinstance(metric, MeanMetric)
                loss = metric.compute()  # NaN when this dataset saw no batch in the current (subset) loop
                if not torch.isnan(loss):
                    out[f"eval/{label}/CrossEntropyLoss"] = loss.item()
                    out[f"eval/{label}/Perplexity"] = torch.exp(loss).item()
            return out
        raise ValueError(f"Unexpected evaluator type '{self.type}'")

    def update_metrics(self, batch: Dict[str, Any], ce_loss: torch.Tensor, logits: torch.Tensor) -> None:
        if self.type == EvaluatorType.downstream:
            assert isinstance(self.eval_metric, ICLMetric)
            self.eval_metric.update(batch, logits)
        elif self.type == EvaluatorType.lm:
            for metadata, instance_loss in zip(batch["metadata"], ce_loss):
                metric = self.eval_metric[metadata["label"]] if isinstance(self.eval_metric, dict) else self.eval_metric
                metric.update(instance_loss)  # type: ignore[union-attr]
        else:
            raise ValueError(f"Unexpected evaluator type '{self.type}'")
