"""Batch assembly with left/right padding (reference: ``olmo/data/collator.py:14-174``)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Union

import torch
import torch.nn.functional as F

from ..config import PaddingDirection, TrainConfig

__all__ = ["DataCollator", "CustomDatasetDataCollator"]


def _as_tensor(x: Any) -> torch.Tensor:
    return x if isinstance(x, torch.Tensor) else torch.tensor(x)


@dataclass
class DataCollator:
    pad_direction: PaddingDirection
    pad_token_id: int

    @classmethod
    def from_train_config(cls, config: TrainConfig) -> "DataCollator":
        return cls(pad_direction=config.data.pad_direction, pad_token_id=config.model.pad_token_id)

    def __call__(self, items: Union[List[Dict[str, Any]], List[torch.Tensor]]) -> Dict[str, Any]:
        assert items
        rows = [x if isinstance(x, dict) else {"input_ids": x} for x in items]
        max_len = max(len(r["input_ids"]) for r in rows)
        max_docs = max((len(r["doc_lens"]) for r in rows if r.get("doc_lens") is not None), default=0)
        cols: Dict[str, List[Any]] = {k: [] for k in (
            "input_ids", "attention_mask", "attention_bias", "label_mask", "index", "instance_mask", "doc_lens", "max_doc_lens", "metadata",
        )}
        for r in rows:
            ids = _as_tensor(r["input_ids"])
            gap = max_len - len(ids)
            pad = (gap, 0) if self.pad_direction == PaddingDirection.left else (0, gap)
            cols["input_ids"].append(F.pad(ids.to(dtype=torch.long), pad, value=self.pad_token_id))
            if (am := r.get("attention_mask")) is not None:
                cols["attention_mask"].append(F.pad(_as_tensor(am).to(dtype=torch.float), pad, value=0.0))
            if (ab := r.get("attention_bias")) is not None:
                ab = _as_tensor(ab)
                while ab.dim() < 3:
                    ab = ab.unsqueeze(0)
                fill = False if ab.dtype == torch.bool else float("-inf")
                cols["attention_bias"].append(F.pad(ab, pad + pad, value=fill))
            if (lm := r.get("label_mask")) is not None:
                cols["label_mask"].append(F.pad(_as_tensor(lm).to(dtype=torch.bool), pad, value=False))
            if (idx := r.get("index")) is not None:
                cols["index"].append(torch.tensor(idx))
            if (im := r.get("instance_mask")) is not None:
                cols["instance_mask"].append(torch.tensor(im))
            if (dl := r.get("doc_lens")) is not None:
                dl = _as_tensor(dl)
                cols["doc_lens"].append(F.pad(dl, (0, max_docs - len(dl)), value=0))
                cols["max_doc_lens"].append(int(dl.max()))
            if (md := r.get("metadata")) is not None:
                cols["metadata"].append(md)
        out: Dict[str, Any] = {}
        for key, values in cols.items():
            if not values:
                continue
            out[key] = values if key in ("max_doc_lens", "metadata") else torch.stack(values)
        return out


@dataclass
class CustomDatasetDataCollator(DataCollator):
    """Collator for user datasets whose items use other field names."""

    input_id_field: str = "input_ids"
    attention_mask_field: Optional[str] = None
    attention_bias_field: Optional[str] = None
    label_mask_field: Optional[str] = None
    index_field: Optional[str] = None
    instance_mask_field: Optional[str] = None
    doc_lens_field: Optional[str] = None
    metadata_field: Optional[str] = None

    def _relabel_item(self, item: Dict[str, Any]) -> Dict[str, Any]:
        def pick(name: Optional[str]):
            return item[name] if name else None

        out = {
            "input_ids": item[self.input_id_field],
            "attention_mask": pick(self.attention_mask_field),
            "attention_bias": pick(self.attention_bias_field),
            "label_mask": pick(self.label_mask_field),
            "index": pick(self.index_field),
            "instance_mask": pick(self.instance_mask_field),
            "metadata": pick(self.metadata_field),
        }
        if self.doc_lens_field:
            out["doc_lens"] = item[self.doc_lens_field]
        return out

    def __call__(self, items: Union[List[Dict[str, Any]], List[torch.Tensor]]) -> Dict[str, Any]:
        if not isinstance(items[0], torch.Tensor):
            items = [self._relabel_item(x) for x in items]  # type: ignore[arg-type]
        return super().__call__(items)
