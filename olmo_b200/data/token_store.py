"""
Positional access to the whole chunks of a list of flat token files.

``TokenStore`` is the layer under :class:`olmo_b200.data.MemMapDataset`: it knows how many whole chunks every file holds,
maps a global instance number to ``(file, chunk)`` with one vectorised search, and reads *batches* of chunks.  Local
files are read by the C++ reader in ``csrc/cpu/token_gather.cpp`` (threads + ``pread`` + in-place widening to int64,
optionally straight into pinned memory); remote files, and machines without a C++ compiler, use byte-range requests from
a thread pool.  Both paths return the same tensors.
"""
from __future__ import annotations

import ctypes
import hashlib
import logging
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from ..aliases import PathOrStr
from ..util import file_size, get_bytes_range, is_url

__all__ = ["TokenStore", "native_reader_available"]

log = logging.getLogger(__name__)

_PKG = Path(__file__).resolve().parent.parent
_SRC = _PKG / "csrc" / "cpu" / "token_gather.cpp"
_SO = _PKG / "_token_gather.so"
_STAMP = _PKG / "_token_gather.stamp"
_lib: Optional[ctypes.CDLL] = None
_lib_failed = False


def _load_native() -> Optional[ctypes.CDLL]:
    """Build (once per source change) and load the C++ reader; ``None`` when that is not possible here."""
    global _lib, _lib_failed
    if _lib is not None or _lib_failed:
        return _lib
    if os.environ.get("OLMO_B200_NATIVE_DATA", "1").strip().lower() in ("0", "false", "no", "off"):
        _lib_failed = True
        return None
    try:
        digest = hashlib.sha256(_SRC.read_bytes()).hexdigest()
        if not (_SO.exists() and _STAMP.exists() and _STAMP.read_text().strip() == digest):
            cxx = shutil.which("g++") or shutil.which("c++")
            if cxx is None:
                raise OSError("no C++ compiler")
            tmp = _SO.with_suffix(f".so.tmp{os.getpid()}")
            proc = subprocess.run([cxx, "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", str(_SRC), "-o", str(tmp)],
                                  stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
            if proc.returncode != 0:
                raise OSError(proc.stdout)
            os.replace(tmp, _SO)
            _STAMP.write_text(digest)
        lib = ctypes.CDLL(str(_SO))
        lib.ob_token_store_open.restype = ctypes.c_void_p
        lib.ob_token_store_open.argtypes = [ctypes.POINTER(ctypes.c_char_p), ctypes.c_int]
        lib.ob_token_store_close.argtypes = [ctypes.c_void_p]
        lib.ob_token_store_read.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
        _lib = lib
    except OSError as e:
        log.warning("native token reader unavailable (%s); using byte-range reads", str(e).strip().splitlines()[-1] if str(e).strip() else e)
        _lib_failed = True
    return _lib


def native_reader_available() -> bool:
    return _load_native() is not None


class TokenStore:
    """Whole chunks of ``chunk`` tokens over ``paths`` (dtype ``dtype``), addressed ``0 .. len(store) - 1``.

    The tail of a file that does not fill a chunk is not addressable, and a file shorter than one chunk contributes
    nothing (but keeps its position, so ``file_of`` indexes ``paths``).
    """

    def __init__(self, paths: Sequence[PathOrStr], dtype, chunk: int, threads: int = 8):
        if chunk <= 0:
            raise ValueError("chunk must be positive")
        self.paths: List[str] = [str(p) for p in paths]
        self.dtype = np.dtype(dtype)
        self.chunk = int(chunk)
        self.threads = int(threads)
        self._ends: Optional[np.ndarray] = None  # cumulative chunk counts, one entry per file
        self._handle: Optional[int] = None
        self._local = all(not is_url(p) for p in self.paths)

    # ------------------------------------------------------------------ extent table
    @property
    def chunk_bytes(self) -> int:
        return self.chunk * self.dtype.itemsize

    def chunks_per_file(self) -> np.ndarray:
        ends = self._extents()
        return np.diff(ends, prepend=0)

    def _extents(self) -> np.ndarray:
        if self._ends is None:
            with ThreadPoolExecutor(max_workers=min(32, max(1, len(self.paths)))) as pool:
                sizes = list(pool.map(file_size, self.paths))
            counts = np.asarray([s // self.chunk_bytes for s in sizes], dtype=np.int64)
            self._ends = np.cumsum(counts)
        return self._ends

    def __len__(self) -> int:
        ends = self._extents()
        return int(ends[-1]) if len(ends) else 0

    def file_ranges(self) -> List[Tuple[int, int]]:
        """``(first instance, one past the last)`` per file."""
        ends = self._extents()
        starts = np.concatenate([[0], ends[:-1]]) if len(ends) else ends
        return [(int(a), int(b)) for a, b in zip(starts, ends)]

    def locate(self, instances) -> Tuple[np.ndarray, np.ndarray]:
        """``(file index, chunk index inside that file)`` for an array of instance numbers (negative numbers count from the end)."""
        idx = np.asarray(instances, dtype=np.int64).reshape(-1)
        n = len(self)
        idx = np.where(idx < 0, idx + n, idx)
        if idx.size and (idx.min() < 0 or idx.max() >= n):
            bad = int(np.asarray(instances).reshape(-1)[np.argmax((idx < 0) | (idx >= n))])
            raise IndexError(f"{bad} is out of bounds for dataset of size {n}")
        ends = self._extents()
        files = np.searchsorted(ends, idx, side="right")  # first file whose cumulative count exceeds the instance: empty files are skipped
        starts = np.where(files > 0, ends[np.maximum(files - 1, 0)], 0)
        return files.astype(np.int32), idx - starts

    # ------------------------------------------------------------------------- reads
    def _native(self) -> Optional[ctypes.CDLL]:
        if not self._local:
            return None
        lib = _load_native()
        if lib is not None and self._handle is None:
            arr = (ctypes.c_char_p * len(self.paths))(*[p.encode() for p in self.paths])
            self._handle = lib.ob_token_store_open(arr, len(self.paths))
        return lib if self._handle else None

    def read(self, instances, out: Optional[torch.Tensor] = None, pin_memory: bool = False) -> torch.Tensor:
        """``[n, chunk] int64`` tokens of the given instances, in the given order (``out``: a preallocated destination)."""
        files, chunks = self.locate(instances)
        n = files.shape[0]
        if out is None:
            out = torch.empty((n, self.chunk), dtype=torch.int64, pin_memory=pin_memory and torch.cuda.is_available())
        assert out.shape == (n, self.chunk) and out.dtype == torch.int64 and out.is_contiguous() and not out.is_cuda
        if n == 0:
            return out
        lib = self._native()
        if lib is not None:
            failed = ctypes.c_int64(-1)
            files_c, chunks_c = np.ascontiguousarray(files), np.ascontiguousarray(chunks)
            rc = lib.ob_token_store_read(self._handle, files_c.ctypes.data, chunks_c.ctypes.data, n, self.chunk, self.dtype.itemsize,
                                         out.data_ptr(), self.threads, ctypes.byref(failed))
            if rc != 0:
                where = self.paths[int(files[failed.value])] if failed.value >= 0 else "?"
                raise OSError(f"reading tokens failed (code {rc}) at {where}")
            return out

        def fetch(i: int) -> None:
            raw = get_bytes_range(self.paths[int(files[i])], int(chunks[i]) * self.chunk_bytes, self.chunk_bytes)
            out[i] = torch.from_numpy(np.frombuffer(raw, dtype=self.dtype).astype(np.int64))

        if n <= 1 or self.threads <= 1:
            for i in range(n):
                fetch(i)
        else:
            with ThreadPoolExecutor(max_workers=min(self.threads, n)) as pool:
                list(pool.map(fetch, range(n)))
        return out

    def close(self) -> None:
        if self._handle is not None and _lib is not None:
            _lib.ob_token_store_close(self._handle)
        self._handle = None

    def __del__(self):  # noqa: D105
        try:
            self.close()
        except Exception:
            pass

    def __getstate__(self):
        state = self.__dict__.copy()
        state["_handle"] = None  # descriptors are per process: data-loader workers reopen
        return state
