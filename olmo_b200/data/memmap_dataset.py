"""
Fixed-length instances over concatenated flat token files (reference: ``olmo/data/memmap_dataset.py:20-247``).

Files are headerless little-endian arrays of ``memmap_dtype`` tokens; instance ``i`` is tokens
``[i·chunk, (i+1)·chunk)`` of the concatenation of whole chunks of every file.  Reads are byte-range requests, so
local paths and every registered URL scheme work alike.  File sizes are resolved once, lazily, in a thread pool.
"""
from __future__ import annotations

import bisect
from concurrent.futures import ThreadPoolExecutor
from copy import deepcopy
from typing import Any, Dict, List, Optional, Tuple, Type, Union

import numpy as np
import torch
from torch.utils.data import Dataset

from ..aliases import PathOrStr
from ..config import InstanceFilterConfig
from ..util import file_size, get_bytes_range
from .util import find_periodic_sequences, get_document_lengths

__all__ = ["MemMapDataset"]


class MemMapDataset(Dataset[Dict[str, Any]]):
    def __init__(
        self,
        *paths: PathOrStr,
        chunk_size: int = 1024,
        memmap_dtype: Union[Type[np.uint8], Type[np.uint16], Type[np.uint32], Type[np.uint64]] = np.uint16,
        metadata: Optional[Union[List[Dict[str, Any]], Dict[str, Any]]] = None,
        include_instance_metadata: bool = True,
        generate_attention_mask: bool = False,
        generate_doc_lengths: bool = False,
        pad_token_id: Optional[int] = None,
        eos_token_id: Optional[int] = None,
        label_mask_paths: Optional[List[PathOrStr]] = None,
        instance_filter_config: Optional[InstanceFilterConfig] = None,
    ):
        if not paths:
            raise ValueError("At least one path is required")
        if generate_attention_mask and pad_token_id is None:
            raise ValueError("'pad_token_id' is required for 'generate_attention_mask'")
        if generate_doc_lengths and eos_token_id is None:
            raise ValueError("'eos_token_id' is required for 'generate_cu_doc_lengths'")
        if label_mask_paths and len(label_mask_paths) != len(paths):
            raise ValueError("There must be the same number of 'label_mask_paths' as there are 'paths'")
        if isinstance(metadata, list):
            if len(metadata) != len(paths):
                raise ValueError("'metadata' should have the same length as the number of file paths")
        else:
            metadata = [metadata or {}] * len(paths)
        self._memmap_paths = paths
        self._metadata = metadata
        self._label_mask_paths = label_mask_paths
        self._chunk_size = chunk_size
        self._mmap_offsets: Optional[List[Tuple[int, int]]] = None
        self._starts: List[int] = []
        self.dtype = memmap_dtype
        self._include_instance_metadata = include_instance_metadata
        self._generate_attention_mask = generate_attention_mask
        self._generate_doc_lengths = generate_doc_lengths
        self._pad_token_id = pad_token_id
        self._eos_token_id = eos_token_id
        self.instance_filter_config = instance_filter_config

    @property
    def chunk_size(self) -> int:
        return self._chunk_size

    @property
    def max_seq_len(self) -> int:
        return self._chunk_size

    def _chunks_in(self, path: PathOrStr, dtype) -> int:
        return file_size(path) // (np.dtype(dtype).itemsize * self._chunk_size)

    @property
    def offsets(self) -> List[Tuple[int, int]]:
        """``(first instance, one past last instance)`` of every file."""
        if self._mmap_offsets is None:
            with ThreadPoolExecutor() as pool:
                lengths = list(pool.map(lambda p: self._chunks_in(p, self.dtype), self._memmap_paths))
                mask_lengths = (
                    list(pool.map(lambda p: self._chunks_in(p, np.bool_), self._label_mask_paths))
                    if self._label_mask_paths is not None
                    else None
                )
            if mask_lengths is not None:
                for path, mpath, a, b in zip(self._memmap_paths, self._label_mask_paths, lengths, mask_lengths):  # type: ignore[arg-type]
                    if a != b:
                        raise ValueError(f"masking file '{mpath}' should be the same size as '{path}'")
            offsets, start = [], 0
            for n in lengths:
                offsets.append((start, start + n))
                start += n
            self._mmap_offsets = offsets
            self._starts = [o[0] for o in offsets]
        return self._mmap_offsets

    def _read_chunk(self, path: PathOrStr, index: int, dtype=None) -> torch.Tensor:
        dtype = dtype or self.dtype
        nbytes = np.dtype(dtype).itemsize * self._chunk_size
        array = np.frombuffer(get_bytes_range(path, index * nbytes, nbytes), dtype=dtype)
        if dtype == np.bool_:
            return torch.tensor(array)
        return torch.tensor(array.astype(np.int_), dtype=torch.long)

    def __len__(self) -> int:
        return self.offsets[-1][1]

    def __getitem__(self, index: int) -> Dict[str, Any]:
        index = int(index)
        n = len(self)
        pos = index if index >= 0 else n + index
        if not 0 <= pos < n:
            raise IndexError(f"{index} is out of bounds for dataset of size {n}")
        file_idx = bisect.bisect_right(self._starts, pos) - 1
        while self.offsets[file_idx][1] <= pos:  # skip files that contribute no whole chunk
            file_idx += 1
        local = pos - self.offsets[file_idx][0]
        input_ids = self._read_chunk(self._memmap_paths[file_idx], local)
        out: Dict[str, Any] = {"input_ids": input_ids}
        if self.instance_filter_config is not None:
            out["instance_mask"] = self._validate_instance(input_ids)
        if self._label_mask_paths is not None:
            out["label_mask"] = self._read_chunk(self._label_mask_paths[file_idx], local, dtype=np.bool_)
        if self._include_instance_metadata:
            out["metadata"] = deepcopy(self._metadata[file_idx])
        if self._generate_attention_mask:
            mask = torch.ones_like(input_ids)
            mask.masked_fill_(input_ids == self._pad_token_id, 0)
            out["attention_mask"] = mask
        if self._generate_doc_lengths:
            out["doc_lens"] = get_document_lengths(input_ids, self._eos_token_id)  # type: ignore[arg-type]
        return out

    def __add__(self, other: "MemMapDataset") -> "MemMapDataset":
        if not isinstance(other, MemMapDataset):
            raise NotImplementedError(f"Expected another MemMapDataset but got {type(other)}")
        return MemMapDataset(
            *(self._memmap_paths + other._memmap_paths),
            chunk_size=self._chunk_size,
            memmap_dtype=self.dtype,
            metadata=self._metadata + other._metadata,
        )

    def _validate_instance(self, input_ids: torch.Tensor) -> bool:
        """False when some short pattern repeats ``repetition_max_count`` times or more (degenerate text)."""
        cfg = self.instance_filter_config
        if cfg is None:
            return True
        for m in find_periodic_sequences(input_ids.numpy(), max_period=cfg.repetition_max_period, min_period=cfg.repetition_min_period):
            if m.times >= cfg.repetition_max_count:
                return False
        return True
