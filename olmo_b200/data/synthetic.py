"""
Seeded synthetic token data for benchmarks and plumbing tests (no counterpart in the reference, which always
reads tokenised corpora).

Instance ``i`` is a pure function of ``(seed, i)``: tokens i.i.d. uniform over ``[0, vocab_size)`` with an EOS
token inserted at geometric(``1/mean_doc_len``) document boundaries, so any rank or restart regenerates the same data.
"""
from __future__ import annotations

from typing import Any, Dict, Optional

import numpy as np
import torch
from torch.utils.data import Dataset

__all__ = ["SyntheticTokenDataset"]


class SyntheticTokenDataset(Dataset[Dict[str, Any]]):
    def __init__(self, num_instances: int, seq_len: int, vocab_size: int, eos_token_id: int, seed: int = 0, mean_doc_len: int = 256):
        self.num_instances, self.seq_len = num_instances, seq_len
        self.vocab_size, self.eos_token_id = vocab_size, eos_token_id
        self.seed, self.mean_doc_len = seed, mean_doc_len

    def __len__(self) -> int:
        return self.num_instances

    def __getitem__(self, index: int) -> Dict[str, Any]:
        index = int(index)
        if not 0 <= index < self.num_instances:
            raise IndexError(index)
        rng = np.random.Generator(np.random.PCG64([self.seed, index]))
        ids = rng.integers(0, self.vocab_size, size=self.seq_len, dtype=np.int64)
        if self.mean_doc_len > 0:
            ids[rng.random(self.seq_len) < 1.0 / self.mean_doc_len] = self.eos_token_id
        return {"input_ids": torch.from_numpy(ids)}

    def batch(self, first: int, count: int, pin: bool = False) -> torch.Tensor:
        """``count`` consecutive instances as one ``(count, seq_len)`` int64 tensor (optionally in pinned memory)."""
        out = torch.empty((count, self.seq_len), dtype=torch.int64, pin_memory=pin)
        for j in range(count):
            out[j] = self[(first + j) % self.num_instances]["input_ids"]
        return out
