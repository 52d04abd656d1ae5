"""
Process-group and device helpers (reference: ``olmo/torch_util.py:11-171``).

All rank queries work without an initialised process group (they fall back to the launcher's
environment variables, then to rank 0 / world 1), which is what lets the same code run under
``torchrun`` over NCCL, as Gloo ranks on CPU, or as a single process.
"""
from __future__ import annotations

import gc
import os
from typing import Any, Optional, TypeVar

import torch
import torch.distributed as dist

T = TypeVar("T")

__all__ = [
    "nvtx_range",
    "seed_all",
    "is_distributed",
    "get_node_rank",
    "get_world_size",
    "get_local_world_size",
    "get_global_rank",
    "get_local_rank",
    "get_fs_local_rank",
    "move_to_device",
    "ensure_finite_",
    "get_default_device",
    "barrier",
    "peak_gpu_memory",
    "synchronize_value",
    "synchronize_flag",
    "gc_cuda",
    "get_cumulative_document_lengths",
    "SingleAccelerator",
]


def seed_all(seed: int) -> None:
    """Seed python, numpy and torch (all devices)."""
    import random

    import numpy as np

    if not 0 <= seed <= 2**32 - 1:
        raise ValueError(f"Seed {seed} is invalid. It must be on [0; 2^32 - 1]")
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


class _Placement:
    """Where this process sits in the job.  The process group answers when there is one; otherwise the variables the
    launcher exported (``RANK``, ``LOCAL_RANK``, ``LOCAL_WORLD_SIZE``, ``NODE_RANK``); otherwise a job of one."""

    @staticmethod
    def env(name: str, default: Optional[int] = None) -> Optional[int]:
        text = os.environ.get(name, "")
        return int(text) if text != "" else default

    @classmethod
    def world(cls) -> int:
        return dist.get_world_size() if is_distributed() else 1

    @classmethod
    def rank(cls) -> int:
        return dist.get_rank() if is_distributed() else cls.env("RANK", 0)  # type: ignore[return-value]

    @classmethod
    def local_rank(cls) -> int:
        return cls.env("LOCAL_RANK", 0)  # type: ignore[return-value]

    @classmethod
    def local_world(cls) -> int:
        return cls.env("LOCAL_WORLD_SIZE") or 1

    @classmethod
    def node(cls) -> int:
        given = cls.env("NODE_RANK")
        return given if given is not None else (cls.rank() - cls.local_rank()) // cls.local_world()

    @classmethod
    def fs_local_rank(cls) -> int:
        explicit = cls.env("FS_LOCAL_RANK")
        if explicit is not None:
            return explicit
        # one filesystem for the whole job: only global rank 0 is "first on its filesystem"
        return cls.rank() if os.environ.get("OLMO_SHARED_FS") else cls.local_rank()


def get_node_rank() -> int:
    return _Placement.node()


def get_world_size() -> int:
    return _Placement.world()


def get_local_world_size() -> int:
    return _Placement.local_world()


def get_global_rank() -> int:
    return _Placement.rank()


def get_local_rank() -> int:
    return _Placement.local_rank()


def get_fs_local_rank() -> int:
    """Rank among the processes that share this process's filesystem: ``FS_LOCAL_RANK`` when set; the global rank when
    ``OLMO_SHARED_FS`` says every rank sees the same files (so only global rank 0 writes shared artefacts); else the
    local rank."""
    return _Placement.fs_local_rank()


def _map_tensors(o: Any, fn):
    """Apply ``fn`` to every tensor inside nested dicts / lists / tuples; everything else passes through."""
    if isinstance(o, torch.Tensor):
        return fn(o)
    if isinstance(o, dict):
        return {k: _map_tensors(v, fn) for k, v in o.items()}
    if isinstance(o, (list, tuple)):
        return type(o)(_map_tensors(x, fn) for x in o)
    return o


def move_to_device(o: T, device: torch.device) -> T:
    """Move the tensors of a nested batch; ``non_blocking`` so that copies from pinned memory overlap."""
    return _map_tensors(o, lambda t: t.to(device, non_blocking=True))


def ensure_finite_(x: torch.Tensor, check_neg_inf: bool = True, check_pos_inf: bool = False) -> None:
    """Replace ``-inf`` / ``+inf`` in place by the dtype's finite extremes."""
    if check_neg_inf:
        x.masked_fill_(x == float("-inf"), torch.finfo(x.dtype).min)
    if check_pos_inf:
        x.masked_fill_(x == float("inf"), torch.finfo(x.dtype).max)


def get_default_device() -> torch.device:
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        return torch.device("cuda")
    return torch.device("cpu")


def barrier() -> None:
    if is_distributed():
        dist.barrier()


def peak_gpu_memory(reset: bool = False) -> Optional[float]:
    """Peak allocated device memory in MB, maximised over ranks; ``None`` without CUDA."""
    if not torch.cuda.is_available():
        return None
    device = torch.device("cuda")
    peak_mb = torch.cuda.max_memory_allocated(device) / 1_000_000
    if is_distributed():
        t = torch.tensor(peak_mb, device=device)
        dist.reduce(t, 0, dist.ReduceOp.MAX)
        peak_mb = t.item()
    if reset:
        torch.cuda.reset_max_memory_allocated(device)
    return peak_mb


V = TypeVar("V", bool, int, float)


def synchronize_value(value: V, device: torch.device) -> V:
    """Broadcast rank 0's scalar to every rank."""
    if is_distributed():
        t = torch.tensor(value, device=device)
        dist.broadcast(t, 0)
        return t.item()  # type: ignore[return-value]
    return value


def synchronize_flag(flag: bool, device: torch.device) -> bool:
    return synchronize_value(flag, device)


def gc_cuda() -> None:
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


def get_cumulative_document_lengths(doc_lens: torch.Tensor) -> torch.Tensor:
    """``(B, max_docs)`` zero-padded document lengths -> int32 ``cu_seqlens`` with a leading 0."""
    flat = doc_lens.reshape(-1)
    flat = flat[flat != 0]
    out = torch.zeros(flat.numel() + 1, dtype=torch.int32, device=doc_lens.device)
    torch.cumsum(flat, 0, dtype=torch.int32, out=out[1:])
    return out


class SingleAccelerator(torch.nn.Module):
    """Single-device stand-in for a distributed wrapper: exposes ``.module`` and ``process_group=None``."""

    process_group = None

    def __init__(self, module: torch.nn.Module) -> None:
        super().__init__()
        self.module = module

    def forward(self, *args: Any, **kwargs: Any):
        return self.module(*args, **kwargs)


class nvtx_range:
    """``with nvtx_range("name"):`` marks a span for timeline profilers when ``OLMO_B200_NVTX=1`` and the process has a
    GPU; otherwise it does nothing (no import, no call into the driver)."""

    _enabled: Optional[bool] = None

    def __init__(self, name: str):
        self.name = name

    @classmethod
    def enabled(cls) -> bool:
        if cls._enabled is None:
            cls._enabled = os.environ.get("OLMO_B200_NVTX", "0").strip().lower() in ("1", "true", "yes", "on") and torch.cuda.is_available()
        return cls._enabled

    def __enter__(self) -> "nvtx_range":
        if self.enabled():
            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc) -> None:
        if self.enabled():
            torch.cuda.nvtx.range_pop()
