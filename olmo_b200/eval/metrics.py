"""
Metric accumulators with cross-rank synchronisation, written against ``torch.distributed`` directly (the
reference uses ``torchmetrics``; ``olmo/eval/downstream.py:28-165``, ``olmo/eval/evaluator.py``).
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..torch_util import is_distributed

__all__ = ["Metric", "MeanMetric", "ICLMetric"]

LOG_2_OF_E = 1.44269504089


class Metric:
    def __init__(self) -> None:
        self.device = torch.device("cpu")

    def to(self, device) -> "Metric":
        self.device = torch.device(device)
        return self

    def reset(self) -> None:
        raise NotImplementedError

    def compute(self) -> torch.Tensor:
        raise NotImplementedError


class MeanMetric(Metric):
    """Weighted running mean; ``compute`` sums value and weight over all ranks."""

    def __init__(self) -> None:
        super().__init__()
        self.reset()

    def reset(self) -> None:
        self.value = torch.zeros((), dtype=torch.float64)
        self.weight = torch.zeros((), dtype=torch.float64)

    def update(self, value, weight=1.0) -> None:
        v = torch.as_tensor(value, dtype=torch.float64).detach().cpu()
        w = torch.as_tensor(weight, dtype=torch.float64).detach().cpu()
        if w.dim() == 0 and v.dim() > 0:
            w = w.expand_as(v)
        self.value += (v * w).sum()
        self.weight += w.sum()

    def compute(self) -> torch.Tensor:
        pair = torch.stack([self.value, self.weight])
        if is_distributed():
            pair = pair.to(self.device if self.device.type == "cuda" else "cpu")
            dist.all_reduce(pair)
            pair = pair.cpu()
        return (pair[0] / pair[1]).float() if pair[1] != 0 else torch.tensor(float("nan"))


def _binary_f1(labels: List[int], preds: List[int], pos_label: int = 0) -> float:
    tp = sum(1 for l, p in zip(labels, preds) if l == pos_label and p == pos_label)
    fp = sum(1 for l, p in zip(labels, preds) if l != pos_label and p == pos_label)
    fn = sum(1 for l, p in zip(labels, preds) if l == pos_label and p != pos_label)
    return 0.0 if tp == 0 else 2 * tp / (2 * tp + fp + fn)


class ICLMetric(Metric):
    """Ranking metrics for multiple-choice in-context tasks.

    Each (document, continuation) pair contributes one score derived from the continuation's token
    log-likelihoods; per document the highest-scoring continuation is the prediction.
    ``metric_type``: ``acc`` (sum log-lik), ``len_norm`` (per character), ``pmi_dc`` (ratio to a domain-conditional
    run), ``f1`` (binary, positive = continuation 0), ``ce_loss`` (negative per-character log-lik of the single
    scored answer), ``bpb`` (bits per byte).
    """

    def __init__(self, metric_type: str = "acc") -> None:
        super().__init__()
        self.metric_type = metric_type
        self.reset()

    def reset(self) -> None:
        self.scores: List[Tuple[int, int, float]] = []
        self.labels: List[Tuple[int, int, int]] = []

    def update(self, batch: Dict[str, Any], lm_logits: torch.Tensor, dc_lm_logits: Optional[torch.Tensor] = None) -> None:
        logp = F.log_softmax(lm_logits.float(), dim=-1)
        dc_logp = None
        if self.metric_type == "pmi_dc":
            assert dc_lm_logits is not None, "PMI_DC acc type selected but no domain conditional logits provided"
            dc_logp = F.log_softmax(dc_lm_logits.float(), dim=-1)
        for i, (doc_id, cont_id) in enumerate(zip(batch["doc_id"], batch["cont_id"])):
            n = int(batch["cont_len"][i])
            cont = batch["continuation"][i][:n]
            ctx = int(batch["ctx_len"][i])
            # logits at position t predict token t+1, hence the -1
            ll = logp[i, ctx - 1 : ctx + n - 1].gather(1, cont.unsqueeze(-1)).sum()
            kind = self.metric_type
            if kind == "pmi_dc":
                dc = int(batch["dc_len"][i])
                score = ll / dc_logp[i, dc - 1 : dc + n - 1].gather(1, cont.unsqueeze(-1)).sum()  # type: ignore[index]
            elif kind in ("acc", "f1"):
                score = ll
            elif kind in ("len_norm", "ce_loss"):
                score = ll / batch["cont_str_len"][i]
                if kind == "ce_loss":
                    score = -score
            elif kind == "bpb":
                score = -ll / batch["cont_byte_len"][i] * LOG_2_OF_E
            else:
                raise ValueError(kind)
            self.scores.append((int(doc_id), int(cont_id), float(score)))
            self.labels.append((int(doc_id), int(cont_id), int(batch["label_id"][i])))

    def _gathered(self) -> Tuple[List[Tuple[int, int, float]], List[Tuple[int, int, int]]]:
        if not is_distributed():
            return self.scores, self.labels
        bucket: List[Any] = [None] * dist.get_world_size()
        dist.all_gather_object(bucket, (self.scores, self.labels))
        scores = [s for part in bucket for s in part[0]]
        labels = [l for part in bucket for l in part[1]]
        return scores, labels

    def compute(self) -> torch.Tensor:
        scores, labels = self._gathered()
        label_of: Dict[int, int] = {}
        for doc_id, _, label in labels:
            label_of.setdefault(doc_id, label)
        per_doc: Dict[int, Dict[int, float]] = {}
        for doc_id, cont_id, s in scores:  # samplers may duplicate instances to even out ranks: first one wins
            per_doc.setdefault(doc_id, {}).setdefault(cont_id, s)
        correct: List[float] = []
        preds: List[int] = []
        golds: List[int] = []
        for doc_id, conts in per_doc.items():
            k = len(conts)
            if any(c >= k for c in conts):  # some continuation of this document was never scored
                continue
            row = torch.full((k,), -float("inf"))
            for c, s in conts.items():
                row[c] = s
            if self.metric_type in ("ce_loss", "bpb"):
                correct.append(float(row[0]))
            else:
                best = int(torch.argmax(row))
                correct.append(1.0 if best == label_of[doc_id] else 0.0)
                preds.append(best)
                golds.append(label_of[doc_id])
        if self.metric_type == "f1":
            return torch.tensor(_binary_f1(golds, preds, pos_label=0))
        return torch.tensor(sum(correct) / len(correct)) if correct else torch.tensor(float("nan"))
