"""Token-sequence helpers: periodic-run detection for the repetition filter, document lengths
(reference: ``olmo/data/util.py:7-130``)."""
from __future__ import annotations

from typing import Iterator, NamedTuple

import numpy as np
import torch

__all__ = ["RepetitionTuple", "find_periodic_sequences", "get_document_lengths"]


class RepetitionTuple(NamedTuple):
    start: int  # first index of the periodic run
    end: int  # one past its last index
    period: int
    times: int  # complete repetitions inside [start, end)


def find_periodic_sequences(arr: np.ndarray, max_period: int, min_period: int = 1, mask_value: int = -1) -> Iterator[RepetitionTuple]:
    """Yield maximal runs in which ``arr[i] == arr[i + period]`` that repeat at least 3 times.

    For each period ``p`` the boolean vector ``arr[p:] == arr[:-p]`` is scanned for runs of ``True``; a run of length
    ``L`` starting at ``s`` means ``arr[s : s + L + p]`` has period ``p``.
    """
    arr = np.asarray(arr)
    if (arr == mask_value).any():
        raise ValueError("`mask_value` is in the array")
    n = len(arr)
    max_period = min(max_period, n // 3)
    for period in range(min_period, max_period + 1):
        same = arr[period:] == arr[:-period]
        if not same.any():
            continue
        edges = np.diff(np.concatenate(([0], same.view(np.int8), [0])))
        starts, stops = np.flatnonzero(edges == 1), np.flatnonzero(edges == -1)
        for s, e in zip(starts, stops):
            end = int(e) + period
            times = (end - int(s)) // period
            if times > 2:
                yield RepetitionTuple(start=int(s), end=end, period=period, times=times)


def get_document_lengths(input_ids: torch.Tensor, eos_token_id: int) -> torch.Tensor:
    """Lengths of the documents inside one instance; an EOS token closes (and belongs to) its document and a
    trailing partial document counts too."""
    eos = (input_ids == eos_token_id).nonzero(as_tuple=True)[0].to(torch.int32)
    n = input_ids.shape[0]
    bounds = [torch.tensor([-1], dtype=torch.int32), eos]
    if n > 0 and input_ids[-1] != eos_token_id:
        bounds.append(torch.tensor([n - 1], dtype=torch.int32))
    b = torch.cat(bounds)
    return b[1:] - b[:-1]
