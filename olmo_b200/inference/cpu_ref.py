"""ctypes face of the C++ CPU int4 reference (``csrc/cpu/int4_ref.cpp``), built on demand with ``g++`` into
``olmo_b200/_cpu_ref.so`` (no CUDA dependency, so it loads on machines without a GPU)."""
from __future__ import annotations

import ctypes
import hashlib
import os
import shutil
import subprocess
from pathlib import Path
from typing import Optional

import torch

from ..exceptions import OLMoEnvironmentError

_ROOT = Path(__file__).resolve().parent.parent
_SRC = _ROOT / "csrc" / "cpu" / "int4_ref.cpp"
_SO = _ROOT / "_cpu_ref.so"
_STAMP = _ROOT / "_cpu_ref.stamp"
_lib: Optional[ctypes.CDLL] = None


def build(force: bool = False) -> Path:
    digest = hashlib.sha256(_SRC.read_bytes()).hexdigest()
    if not force and _SO.exists() and _STAMP.exists() and _STAMP.read_text().strip() == digest:
        return _SO
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise OLMoEnvironmentError("a C++ compiler is needed to build the CPU int4 reference")
    tmp = _SO.with_suffix(".so.tmp")
    proc = subprocess.run([cxx, "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", str(_SRC), "-o", str(tmp)],
                          stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise OLMoEnvironmentError(f"building {_SRC.name} failed:\n{proc.stdout}")
    os.replace(tmp, _SO)
    _STAMP.write_text(digest)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
    return _lib


def _p(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _host(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Contiguous host copy: the C++ code dereferences the pointer, so a device tensor must never reach it."""
    return t.detach().to(device="cpu", dtype=dtype).contiguous()


def dequant(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, group: int, threads: int = 8) -> torch.Tensor:
    """``[N, K]`` fp32 weights (stored column order) from the packed representation (CPU tensors)."""
    n, k = qweight.shape[0], qweight.shape[1] * 8
    q, s, z = _host(qweight, torch.int32), _host(scales, torch.float32), _host(zeros, torch.uint8)
    out = torch.empty(n, k, dtype=torch.float32)
    rc = lib().ob_cpu_w4a16_dequant(_p(q), _p(s), _p(z), _p(out), n, k, group, threads)
    if rc != 0:
        raise ValueError(f"ob_cpu_w4a16_dequant rejected the shapes (code {rc})")
    return out


def matmul(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, group: int,
           perm: Optional[torch.Tensor] = None, threads: int = 8) -> torch.Tensor:
    """``x[M, K] · Wᵀ`` in fp32 on the CPU."""
    n, k = qweight.shape[0], qweight.shape[1] * 8
    x2 = _host(x.reshape(-1, k), torch.float32)
    q, s, z = _host(qweight, torch.int32), _host(scales, torch.float32), _host(zeros, torch.uint8)
    pm = None if perm is None else _host(perm, torch.int32)
    y = torch.empty(x2.shape[0], n, dtype=torch.float32)
    rc = lib().ob_cpu_w4a16_matmul(_p(x2), _p(q), _p(s), _p(z), _p(pm), _p(y), x2.shape[0], n, k, group, threads)
    if rc != 0:
        raise ValueError(f"ob_cpu_w4a16_matmul rejected the shapes (code {rc})")
    return y.reshape(*x.shape[:-1], n)
