"""
Deterministic, restartable, rank-strided iteration over a map-style dataset
(reference: ``olmo/data/iterable_dataset.py:20-191``).

The global order is one permutation of all instances drawn from ``PCG64(seed + epoch)``, padded (or truncated with
``drop_last``) to a multiple of the world size.  It can be persisted as ``work_dir/global_indices.npy`` (uint32
memmap written by filesystem-local rank 0) so that every rank and every restart reads the same order.  A restart
sets ``start_index`` (instances already consumed globally); rank ``r`` then takes every ``world_size``-th index.
With DataLoader workers each worker takes whole device batches in turn, so batches come out in order.
"""
from __future__ import annotations

import dataclasses
import logging
import math
from pathlib import Path
from typing import Any, Dict, Iterator, List, Optional, Sequence, Union

import numpy as np
import torch
import torch.utils.data

from ..aliases import PathOrStr
from ..torch_util import barrier, get_fs_local_rank, get_global_rank, get_world_size
from ..util import roundrobin, threaded_generator

__all__ = ["IterableDataset"]

log = logging.getLogger(__name__)


class IterableDataset(torch.utils.data.IterableDataset[Dict[str, Any]]):
    def __init__(
        self,
        dataset: Union[Sequence[List[int]], Sequence[torch.Tensor], Sequence[Dict[str, Any]]],
        global_batch_size: int,
        *,
        seed: int = 0,
        epoch: int = 0,
        start_index: int = 0,
        max_examples: Optional[int] = None,
        shuffle: bool = True,
        drop_last: bool = False,
        world_size: Optional[int] = None,
        rank: Optional[int] = None,
        fs_local_rank: Optional[int] = None,
        work_dir: Optional[PathOrStr] = None,
        num_threads: Optional[int] = None,
    ):
        self.dataset = dataset
        self.seed, self.epoch = seed, epoch
        self.start_index = start_index
        self.max_examples = max_examples
        self.shuffle, self.drop_last = shuffle, drop_last
        self.rank = get_global_rank() if rank is None else rank
        self.fs_local_rank = get_fs_local_rank() if fs_local_rank is None else fs_local_rank
        self.world_size = get_world_size() if world_size is None else world_size
        n, w = len(self.dataset), self.world_size  # type: ignore[arg-type]
        per_rank = math.ceil((n - w) / w) if (drop_last and n % w != 0) else math.ceil(n / w)
        self.total_size = per_rank * w
        self.num_threads = num_threads
        assert global_batch_size % w == 0
        self.device_batch_size = global_batch_size // w
        self.global_indices_file: Optional[Path] = None
        self.work_dir = work_dir
        if work_dir is not None:
            self._build_and_save_global_indices()

    def _build_global_indices(self) -> np.ndarray:
        n = len(self.dataset)  # type: ignore[arg-type]
        assert n < np.iinfo(np.uint32).max
        order = np.arange(n, dtype=np.uint32)
        if self.shuffle:
            np.random.Generator(np.random.PCG64(seed=self.seed + self.epoch)).shuffle(order)
        if self.drop_last:
            order = order[: self.total_size]
        elif self.total_size > n:
            reps = math.ceil(self.total_size / n)
            order = np.concatenate([order] * reps)[: self.total_size]  # wrap around to fill the last stride
        assert len(order) == self.total_size
        return order

    def _build_and_save_global_indices(self) -> None:
        assert self.work_dir is not None
        self.global_indices_file = Path(self.work_dir) / "global_indices.npy"
        if self.fs_local_rank == 0:
            log.info("Saving global data order indices...")
            self.global_indices_file.parent.mkdir(parents=True, exist_ok=True)
            order = self._build_global_indices()
            mm = np.memmap(self.global_indices_file, dtype=np.uint32, mode="w+", shape=(len(order),))
            mm[:] = order
            mm.flush()
            del mm
            log.info("Global data order indices saved to '%s'", self.global_indices_file)
        barrier()

    def get_global_indices(self) -> np.ndarray:
        if self.global_indices_file is not None:
            return np.memmap(self.global_indices_file, mode="r", dtype=np.uint32)  # type: ignore[return-value]
        return self._build_global_indices()

    def reshuffle(self, epoch: int) -> None:
        self.epoch = epoch
        if self.work_dir is not None:
            self._build_and_save_global_indices()

    def _my_indices(self) -> np.ndarray:
        """This rank's (and, inside a data-loader worker, this worker's) slice of the global order, in yield order."""
        order = self.get_global_indices()
        if self.max_examples is not None:
            assert self.max_examples % self.world_size == 0
            order = order[: self.max_examples]
        mine = order[self.start_index :][self.rank : self.total_size : self.world_size]
        info = torch.utils.data.get_worker_info()
        if info is None:
            return mine
        # workers take whole device batches in turn (so that the loader emits batches in order); what does not fill a
        # batch is dealt out instance by instance
        bs = self.device_batch_size
        whole = bs * (len(mine) // bs)
        batches = mine[:whole].reshape((-1, bs))[info.id :: info.num_workers].reshape((-1,))
        return np.concatenate([batches, mine[whole + info.id :: info.num_workers]])

    def _batched_items(self, indices: np.ndarray) -> Iterator[Dict[str, Any]]:
        """One batched fetch per device batch (the dataset reads all chunks of a batch in one native call)."""
        bs = self.device_batch_size
        for a in range(0, len(indices), bs):
            ids = [int(i) for i in indices[a : a + bs]]
            for idx, item in zip(ids, self.dataset.__getitems__(ids)):  # type: ignore[union-attr]
                yield self._as_item(item, idx)

    def __iter__(self) -> Iterator[Dict[str, Any]]:
        indices = self._my_indices()
        num_threads = self.num_threads
        if num_threads is None and torch.utils.data.get_worker_info() is None:
            num_threads = 4
        if hasattr(self.dataset, "__getitems__"):
            # the parallelism is inside the batched read; one background thread keeps two batches ahead of the consumer
            items = self._batched_items(indices)
            return threaded_generator(items, maxsize=2 * self.device_batch_size, thread_name="data prefetch") if num_threads else items
        if not num_threads:
            return (self._get_dataset_item(int(i)) for i in indices)
        depth = math.ceil(self.device_batch_size * 2 / num_threads)
        lanes = [
            threaded_generator(
                (self._get_dataset_item(int(i)) for i in indices[t::num_threads]), maxsize=depth, thread_name=f"data thread {t}"
            )
            for t in range(num_threads)
        ]
        return (x for x in roundrobin(*lanes))

    @staticmethod
    def _as_item(item: Any, idx: int) -> Dict[str, Any]:
        if isinstance(item, dict):
            return {**item, "index": idx}
        if dataclasses.is_dataclass(item):
            return dict(**dataclasses.asdict(item), index=idx)  # type: ignore[arg-type]
        return {"input_ids": item, "index": idx}

    def _get_dataset_item(self, idx: int) -> Dict[str, Any]:
        return self._as_item(self.dataset[idx], idx)
