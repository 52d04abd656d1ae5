"""
Fixed-length training instances over flat token files (the dataset the reference defines in
``olmo/data/memmap_dataset.py:20-247``; same constructor and item keys, so configs and downstream code are unchanged).

Files are headerless little-endian arrays of ``memmap_dtype`` tokens; instance ``i`` is the ``i``-th whole chunk of
``chunk_size`` tokens of the files laid end to end (the tail of a file that does not fill a chunk is skipped).  The
dataset is a thin item-assembly layer over :class:`~olmo_b200.data.token_store.TokenStore`, which owns the extent table
and the reads.  Besides ``dataset[i]`` there is the batched ``dataset.__getitems__([...])`` that ``torch``'s data
loader prefers when it exists, and ``dataset.read_batch([...])`` which returns the stacked ``[n, chunk]`` tensors
directly: both fetch all chunks of a batch in one call of the native reader.
"""
from __future__ import annotations

from copy import deepcopy
from typing import Any, Dict, List, Optional, Sequence, Tuple, Type, Union

import numpy as np
import torch
from torch.utils.data import Dataset

from ..aliases import PathOrStr
from ..config import InstanceFilterConfig
from .token_store import TokenStore
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
        n_files = len(paths)
        problems = {
            "At least one path is required": n_files == 0,
            "'pad_token_id' is required for 'generate_attention_mask'": generate_attention_mask and pad_token_id is None,
            "'eos_token_id' is required for 'generate_doc_lengths'": generate_doc_lengths and eos_token_id is None,
            "'label_mask_paths' needs one mask file per token file": bool(label_mask_paths) and len(label_mask_paths or ()) != n_files,
            "'metadata' given as a list needs one entry per token file": isinstance(metadata, list) and len(metadata) != n_files,
        }
        for message, broken in problems.items():
            if broken:
                raise ValueError(message)
        self._memmap_paths = paths
        self._metadata: List[Dict[str, Any]] = metadata if isinstance(metadata, list) else [metadata or {}] * n_files
        self._label_mask_paths = label_mask_paths
        self._chunk_size = chunk_size
        self.dtype = memmap_dtype
        self._tokens = TokenStore(paths, memmap_dtype, chunk_size)
        # label masks are one byte per token in files that line up with the token files
        self._masks = TokenStore(label_mask_paths, np.uint8, chunk_size) if label_mask_paths else None
        self._checked = False
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

    def _check_masks(self) -> None:
        if self._checked:
            return
        if self._masks is not None:
            a, b = self._tokens.chunks_per_file(), self._masks.chunks_per_file()
            for i in np.nonzero(a != b)[0][:1]:
                raise ValueError(f"masking file '{self._label_mask_paths[i]}' should be the same size as '{self._memmap_paths[i]}'")  # type: ignore[index]
        self._checked = True

    @property
    def offsets(self) -> List[Tuple[int, int]]:
        """``(first instance, one past last instance)`` of every file."""
        self._check_masks()
        return self._tokens.file_ranges()

    def __len__(self) -> int:
        self._check_masks()
        return len(self._tokens)

    # ------------------------------------------------------------------------------ access
    def read_batch(self, indices: Sequence[int], pin_memory: bool = False) -> Dict[str, Any]:
        """Stacked tensors for a list of instances: ``input_ids [n, chunk]`` and, where configured, ``label_mask``,
        ``attention_mask``; per-instance values (``metadata``, ``instance_mask``, ``doc_lens``) come as lists."""
        self._check_masks()
        ids = self._tokens.read(indices, pin_memory=pin_memory)
        out: Dict[str, Any] = {"input_ids": ids}
        if self.instance_filter_config is not None:
            out["instance_mask"] = [self._validate_instance(row) for row in ids]
        if self._masks is not None:
            out["label_mask"] = self._masks.read(indices).to(torch.bool)
        if self._include_instance_metadata:
            files, _ = self._tokens.locate(indices)
            out["metadata"] = [deepcopy(self._metadata[int(f)]) for f in files]
        if self._generate_attention_mask:
            out["attention_mask"] = (ids != self._pad_token_id).to(ids.dtype)
        if self._generate_doc_lengths:
            out["doc_lens"] = [get_document_lengths(row, self._eos_token_id) for row in ids]  # type: ignore[arg-type]
        return out

    def __getitems__(self, indices: Sequence[int]) -> List[Dict[str, Any]]:
        batch = self.read_batch(indices)
        return [{key: value[i] for key, value in batch.items()} for i in range(len(indices))]

    def __getitem__(self, index: int) -> Dict[str, Any]:
        return self.__getitems__([int(index)])[0]

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
