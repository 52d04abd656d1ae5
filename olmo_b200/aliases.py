"""Type aliases shared across the package.

``PathOrStr`` is the one the reference exports (``olmo/aliases.py:1-7``); the others name shapes of data that recur
in this package's signatures.
"""
import os
from typing import Any, Dict, Union

import torch

__all__ = ["PathOrStr", "Batch", "StateDict", "Metrics"]

#: A filesystem path, as text or as any ``os.PathLike``; URLs are passed as ``str``.
PathOrStr = Union[str, os.PathLike]

#: One collated batch: ``input_ids`` plus the optional ``attention_mask``, ``label_mask``, ``doc_lens``, ``index``, …
Batch = Dict[str, Any]

#: ``name -> tensor`` (a model's parameters) or the nested dictionary of an optimizer's state.
StateDict = Dict[str, Any]

#: ``logging key -> value`` as produced by a training or evaluation step.
Metrics = Dict[str, Union[float, int, torch.Tensor]]
