"""
Loader and builder of the sm_100a kernel library.

The kernels in ``olmo_b200/csrc`` are compiled by ``nvcc`` into one shared object,
``olmo_b200/_kernels.so``, that exports a plain C interface (``csrc/api.h``) and is opened with
:mod:`ctypes`; tensors cross the boundary as raw device pointers plus the current CUDA stream.
The library is built in-tree (``python -m olmo_b200.ops`` or :func:`build`) and is never replaced by a
silent PyTorch fallback on a GPU machine: :func:`lib` raises if it is missing or stale.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import shutil
import subprocess
import tempfile
from pathlib import Path
from typing import List, Optional

import torch

from ..exceptions import OLMoEnvironmentError, OLMoKernelError

__all__ = ["build", "lib", "available", "require_extension", "enabled", "check_status", "status_tensor", "stream_ptr", "ptr"]

_ROOT = Path(__file__).resolve().parent.parent
_SRC_DIR = _ROOT / "csrc"
_SO_PATH = _ROOT / "_kernels.so"
_STAMP_PATH = _ROOT / "_kernels.stamp"

NVCC_FLAGS: List[str] = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "--use_fast_math",
    "-Xcompiler", "-fPIC", "-shared",
]

_lib: Optional[ctypes.CDLL] = None


def _sources() -> List[Path]:
    return sorted(_SRC_DIR.glob("*.cu"))


def _source_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(_SRC_DIR.glob("*.cu")) + list(_SRC_DIR.glob("*.cuh")) + list(_SRC_DIR.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def is_stale() -> bool:
    return not _SO_PATH.exists() or not _STAMP_PATH.exists() or _STAMP_PATH.read_text().strip() != _source_digest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every ``.cu`` under ``csrc/`` for sm_100a into ``_kernels.so`` (no GPU needed)."""
    global _lib
    if not force and not is_stale():
        return _SO_PATH
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        raise OLMoEnvironmentError("nvcc not found; cannot build the sm_100a kernels")
    objs = []
    # a directory of its own per building process: several ranks that find a stale library at the same time must not
    # write each other's object files (the final rename of the library is atomic)
    (_ROOT / "build").mkdir(exist_ok=True)
    build_dir = Path(tempfile.mkdtemp(prefix=f"p{os.getpid()}_", dir=_ROOT / "build"))
    procs = []
    for src in _sources():
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *[f for f in NVCC_FLAGS if f != "-shared"], "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    for src, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise OLMoEnvironmentError(f"nvcc failed on {src.name}:\n{out}")
        if verbose and out:
            print(out)
    tmp = _SO_PATH.with_suffix(f".so.tmp{os.getpid()}")
    link = subprocess.run(
        [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs), "-o", str(tmp)],
        stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
    )
    if link.returncode != 0:
        raise OLMoEnvironmentError(f"link failed:\n{link.stdout}")
    os.replace(tmp, _SO_PATH)
    _STAMP_PATH.write_text(_source_digest())
    shutil.rmtree(build_dir, ignore_errors=True)
    _lib = None
    return _SO_PATH


def lib() -> ctypes.CDLL:
    """The loaded kernel library.  Raises when it is missing, or stale and cannot be rebuilt."""
    global _lib
    if _lib is None:
        if is_stale():
            if shutil.which("nvcc") or Path("/usr/local/cuda/bin/nvcc").exists():
                build()
            else:
                state = "does not match the sources under csrc/ (stale build)" if _SO_PATH.exists() else "is missing"
                raise OLMoEnvironmentError(f"{_SO_PATH} {state} and nvcc is unavailable; run `python -m olmo_b200.ops` where nvcc exists")
        _lib = ctypes.CDLL(str(_SO_PATH))
        _lib.ob_set_gemm_pair_mode(ctypes.c_int(int(os.environ.get("OLMO_B200_GEMM_2CTA", "1") not in ("0", "", "false"))))
        _lib.ob_set_gemm_tma_store(ctypes.c_int(int(os.environ.get("OLMO_B200_GEMM_TMA_STORE", "1") not in ("0", "", "false"))))
    return _lib


def available() -> bool:
    """True when a CUDA device is present (the kernels target sm_100a only)."""
    return torch.cuda.is_available()


def enabled() -> bool:
    """True when the fused sm_100a path should be used: a GPU is present and the user did not turn it off."""
    if not available():
        return False
    return os.environ.get("OLMO_B200_KERNELS", "1").strip().lower() not in ("0", "false", "no", "off")


def require_extension() -> ctypes.CDLL:
    if not available():
        raise OLMoEnvironmentError("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if major != 10:
        raise OLMoEnvironmentError(f"the kernels are built for sm_100a; found sm_{major}{minor}")
    return lib()


# ------------------------------------------------------------------------------ call helpers

_status = {}


def status_tensor(device: Optional[torch.device] = None) -> torch.Tensor:
    """Per-device int32 status word that kernels with bounded waits write on time-out."""
    idx = torch.cuda.current_device() if device is None or device.index is None else device.index
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status[idx] = t
    return t


def check_status(device: Optional[torch.device] = None) -> None:
    """Synchronising check of the status word; raises :class:`OLMoKernelError` and clears it if non-zero."""
    t = status_tensor(device)
    code = int(t.item())
    if code != 0:
        t.zero_()
        raise OLMoKernelError(f"a device-side bounded wait ran out (status {code})")


def stream_ptr() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


_launches = 0


def check(rc: int, what: str, kernels: int = 1) -> int:
    """Validate a C entry point's return code and count the kernels it launched."""
    global _launches
    if rc < 0:
        raise OLMoKernelError(f"{what} failed to launch (code {rc})")
    _launches += kernels
    return rc


def launch_count() -> int:
    """Number of kernels of this library launched by the current process so far."""
    return _launches
