"""
Offline readers for the sharded checkpoint layouts written by the reference implementation's FSDP1 checkpointers,
so that a run started there can be resumed, unsharded or converted here.  Everything in this module runs in one CPU
process without a process group.

``torch_legacy``  (the reference's default; ``olmo/checkpoint.py:969-1453``)
    ``rank{r}.pt`` per rank, each a ``torch.save`` of ``{"model": {...}, "optim": {...}, **trainer_state}`` in which
    every parameter and every optimizer moment is a ``ShardedTensor``: a pickled object that carries this rank's local
    shards and the table of *all* shards (offsets, sizes, owning rank).  A ``ShardedTensor`` normally refuses to be
    unpickled outside an initialised process group.  The reader below therefore unpickles the files with its own
    ``Unpickler``: the rebuild hook that pickles of tensor subclasses name is swapped, for this load only, for one
    that stores the pickled state of a ``ShardedTensor`` in a plain :class:`ShardedTensorRecord` instead of constructing
    the real object.  Full tensors are then assembled by narrowing to each shard's offsets.

``local``  (``olmo/checkpoint.py:1474-1906``)
    ``metadata.yaml`` (world size), ``model/rank{r}.pt`` with the raw local piece of every FSDP flat parameter plus the
    flat parameter's own tables (names, shapes, and which element range of which parameter the piece covers, in either
    of the two forms torch has used), ``optim/rank{r}.pt`` with the per-parameter optimizer state shards keyed by
    integer id, and ``train/rank{r}.pt``.

``olmo_core``  needs the ``olmo_core`` package's own reader and is reported as unsupported.

The layout of a directory is recognised by :func:`detect_layout`.
"""
from __future__ import annotations

import logging
import pickle
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Iterator, List, Optional, Sequence, Tuple

import torch
import yaml

from .aliases import PathOrStr
from .exceptions import OLMoCheckpointError

__all__ = [
    "ShardedTensorRecord", "detect_layout", "load_with_sharded_tensor_records", "unshard_torch_legacy_checkpoint",
    "unshard_local_checkpoint", "unshard_reference_checkpoint", "export_torch_new_checkpoint",
]

log = logging.getLogger(__name__)

_WRAPPER = "_fsdp_wrapped_module."


def _clean(name: str) -> str:
    return name.replace(_WRAPPER, "")


# ------------------------------------------------------------------------------------------ torch_legacy


@dataclass
class ShardedTensorRecord:
    """What a pickled ``ShardedTensor`` holds: this file's local shards and the global shard table."""

    local_shards: List[Any]  # objects with ``.tensor`` and ``.metadata`` (``shard_offsets``, ``shard_sizes``, ``placement``)
    metadata: Any  # ``ShardedTensorMetadata``: ``shards_metadata``, ``size``, ``tensor_properties``

    @property
    def size(self) -> torch.Size:
        return torch.Size(self.metadata.size)

    @property
    def dtype(self) -> torch.dtype:
        return self.metadata.tensor_properties.dtype


def _record_aware_rebuild(func, new_type, args, state):
    """Stand-in for ``torch._tensor._rebuild_from_type_v2`` used while reading legacy shard files."""
    from torch.distributed._shard.sharded_tensor import ShardedTensor

    if isinstance(new_type, type) and issubclass(new_type, ShardedTensor):
        # pickled state of a ShardedTensor: (local shards, metadata, process-group state, sharding spec, init_rrefs)
        return ShardedTensorRecord(local_shards=list(state[0]), metadata=state[1])
    return torch._tensor._rebuild_from_type_v2(func, new_type, args, state)


class _RecordPickle:
    """A ``pickle_module`` for ``torch.load`` whose unpickler resolves the tensor-subclass rebuild hook to
    :func:`_record_aware_rebuild`.  Nothing global is patched."""

    __name__ = "olmo_b200_record_pickle"

    class Unpickler(pickle.Unpickler):
        def find_class(self, module: str, name: str):  # noqa: D102
            if module == "torch._tensor" and name == "_rebuild_from_type_v2":
                return _record_aware_rebuild
            return super().find_class(module, name)

    @staticmethod
    def load(file, **kwargs):
        return _RecordPickle.Unpickler(file, **kwargs).load()

    loads = staticmethod(pickle.loads)
    dump = staticmethod(pickle.dump)
    dumps = staticmethod(pickle.dumps)
    PickleError = pickle.PickleError
    UnpicklingError = pickle.UnpicklingError
    HIGHEST_PROTOCOL = pickle.HIGHEST_PROTOCOL


def load_with_sharded_tensor_records(path: PathOrStr) -> Any:
    """``torch.load`` of one legacy shard file with every ``ShardedTensor`` replaced by a :class:`ShardedTensorRecord`."""
    return torch.load(str(path), map_location="cpu", weights_only=False, pickle_module=_RecordPickle)


def _shard_rank(shard_md) -> int:
    placement = shard_md.placement
    rank = placement.rank() if hasattr(placement, "rank") else None
    if rank is None:
        text = str(placement)  # "rank:3/cuda:3"
        rank = int(text.split("/")[0].split(":")[1])
    return int(rank)


def _walk(obj: Any, path: Tuple = ()) -> Iterator[Tuple[Tuple, Any]]:
    """Leaves of a nested dict / list structure with their key paths (records and tensors are leaves)."""
    if isinstance(obj, dict):
        for k, v in obj.items():
            yield from _walk(v, path + (k,))
    elif isinstance(obj, (list, tuple)) and not isinstance(obj, torch.Size):
        for i, v in enumerate(obj):
            yield from _walk(v, path + (i,))
    else:
        yield path, obj


def _set(root: Any, path: Tuple, value: Any) -> None:
    cur = root
    for k in path[:-1]:
        cur = cur[k]
    cur[path[-1]] = value


def unshard_torch_legacy_checkpoint(
    load_path: PathOrStr, *, load_optimizer_state: bool = True, load_trainer_state: bool = True,
    device: Optional[torch.device] = None, thread_count: Optional[int] = None,
) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
    """Full model state, optimizer state (keyed by parameter name) and trainer state of a ``torch_legacy`` sharded
    checkpoint.  Rank 0's file provides the skeleton (non-tensor entries, shapes); each file contributes its local
    shards.  A full tensor starts as NaN and every shard listed in the table must arrive, so a missing or truncated
    rank file is an error, not silent garbage."""
    folder = Path(load_path)
    files = sorted(folder.glob("rank*.pt"), key=lambda p: int(p.stem[4:]))
    if not files:
        raise OLMoCheckpointError(f"no rank*.pt files in {folder}")
    ranks = [int(p.stem[4:]) for p in files]
    if ranks != list(range(len(files))):
        raise OLMoCheckpointError(f"rank files in {folder} are not contiguous: {ranks}")
    dev = device or torch.device("cpu")

    def wanted(path: Tuple) -> bool:
        return bool(path) and (path[0] == "model" or (path[0] == "optim" and load_optimizer_state))

    skeleton: Optional[Dict[str, Any]] = None
    full: Dict[Tuple, torch.Tensor] = {}
    remaining: Dict[Tuple, int] = {}

    def absorb(rank: int, state: Dict[str, Any]) -> None:
        for path, leaf in _walk(state):
            if not (wanted(path) and isinstance(leaf, ShardedTensorRecord)):
                continue
            if path not in full:
                full[path] = torch.full(tuple(leaf.size), float("nan"), dtype=leaf.dtype, device=dev)
                remaining[path] = sum(1 for md in leaf.metadata.shards_metadata if _numel(md.shard_sizes) > 0)
            out = full[path]
            for shard in leaf.local_shards:
                md = shard.metadata
                if _shard_rank(md) != rank:
                    raise OLMoCheckpointError(f"{folder}/rank{rank}.pt holds a shard of {path} placed on rank {_shard_rank(md)}")
                if _numel(md.shard_sizes) == 0:
                    continue
                view = out
                for dim, (off, size) in enumerate(zip(md.shard_offsets, md.shard_sizes)):
                    view = view.narrow(dim, off, size)
                view.copy_(shard.tensor.reshape(view.shape))
                remaining[path] -= 1

    with ThreadPoolExecutor(max_workers=thread_count or min(8, len(files))) as pool:
        for rank, state in zip(ranks, pool.map(load_with_sharded_tensor_records, files)):
            if rank == 0:
                skeleton = state
            absorb(rank, state)
            if rank != 0:
                del state
    assert skeleton is not None
    missing = [".".join(map(str, p)) for p, n in remaining.items() if n != 0]
    if missing:
        raise OLMoCheckpointError(f"shards missing for {missing[:5]} (world size of the writing job: {len(files)})")

    for path, tensor in full.items():
        if tensor.is_floating_point() and torch.isnan(tensor).any():
            raise OLMoCheckpointError(f"{'.'.join(map(str, path))} was not fully covered by the shard files")
        _set(skeleton, path, tensor)

    model_state = {_clean(k): v for k, v in skeleton.pop("model").items()}
    optim_raw = skeleton.pop("optim", None)
    optim_state: Optional[Dict[str, Any]] = None
    if load_optimizer_state and optim_raw is not None:
        optim_state = {
            "state": {_clean(str(k)): v for k, v in optim_raw.get("state", {}).items()},
            "param_groups": optim_raw.get("param_groups", []),
        }
        for group in optim_state["param_groups"]:
            for key in ("params", "param_names"):
                if key in group:
                    group[key] = [_clean(n) if isinstance(n, str) else n for n in group[key]]
    skeleton.pop("rng", None)
    trainer_state = {k: v for k, v in skeleton.items()} if load_trainer_state else None
    return model_state, optim_state, trainer_state


def _numel(sizes: Sequence[int]) -> int:
    n = 1
    for s in sizes:
        n *= int(s)
    return n


# ------------------------------------------------------------------------------------------------- local


@dataclass
class _Piece:
    """Element range ``[start, end]`` (inclusive, in the flattened parameter) that one rank holds, and where."""

    shape: torch.Size
    start: int
    end: int
    data: Optional[torch.Tensor]

    def copy_into(self, full: torch.Tensor, data: Optional[torch.Tensor] = None) -> None:
        src = self.data if data is None else data
        assert src is not None
        full.view(-1)[self.start : self.end + 1].copy_(src.reshape(-1))


def _flat_param_pieces(model_state: Dict[str, Any]) -> Iterator[Tuple[str, _Piece]]:
    """``(parameter name, piece)`` for every parameter that has elements in this rank's flat-parameter shards."""
    for module in model_state["modules"]:
        prefix = _clean(module["name"])
        for handle in module["handles"]:
            flat = handle["flat_param.data"]
            fqns, shapes = handle["flat_param._fqns"], handle["flat_param._shapes"]
            if "flat_param._shard_param_infos" in handle:  # torch >= 2.1: one record per parameter of the flat parameter
                for fqn, shape, info in zip(fqns, shapes, handle["flat_param._shard_param_infos"]):
                    in_shard, offset, numel, start, end = tuple(info)[:5]
                    if not in_shard:
                        continue
                    name = fqn if not prefix else f"{prefix}.{fqn}"
                    yield _clean(name), _Piece(torch.Size(shape), int(start), int(end), flat[offset : offset + numel])
            else:  # torch <= 2.0: index range of the parameters present + inclusive element offsets of each
                first = handle["flat_param._shard_indices"][0]
                cursor = 0
                for fqn, shape, (start, end) in zip(fqns[first:], shapes[first:], handle["flat_param._shard_param_offsets"]):
                    n = end - start + 1
                    name = fqn if not prefix else f"{prefix}.{fqn}"
                    yield _clean(name), _Piece(torch.Size(shape), int(start), int(end), flat[cursor : cursor + n])
                    cursor += n


def unshard_local_checkpoint(
    load_path: PathOrStr, *, load_optimizer_state: bool = True, load_trainer_state: bool = True, device: Optional[torch.device] = None,
) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
    """Full states of a ``local`` sharded checkpoint (raw flat-parameter pieces per rank)."""
    folder = Path(load_path)
    meta = yaml.safe_load((folder / "metadata.yaml").read_text()) or {}
    world = int(meta.get("world_size", 0))
    if world <= 0:
        raise OLMoCheckpointError(f"{folder}/metadata.yaml does not give a world size")
    dev = device or torch.device("cpu")
    model_state: Dict[str, torch.Tensor] = {}
    layout: List[Dict[str, _Piece]] = []
    for rank in range(world):
        path = folder / "model" / f"rank{rank}.pt"
        if not path.is_file():
            raise OLMoCheckpointError(f"missing shard file {path}")
        pieces: Dict[str, _Piece] = {}
        for name, piece in _flat_param_pieces(torch.load(path, map_location="cpu", weights_only=False)):
            if name not in model_state:
                model_state[name] = torch.full(tuple(piece.shape), float("nan"), dtype=piece.data.dtype, device=dev)  # type: ignore[union-attr]
            piece.copy_into(model_state[name])
            pieces[name] = _Piece(piece.shape, piece.start, piece.end, None)
        layout.append(pieces)
    for name, tensor in model_state.items():
        if torch.isnan(tensor).any():
            raise OLMoCheckpointError(f"parameter {name} was not fully covered by the shard files")

    trainer_state = None
    if load_trainer_state:
        trainer_state = torch.load(folder / "train" / "rank0.pt", map_location="cpu", weights_only=False)
    if not load_optimizer_state:
        return model_state, None, trainer_state

    state: Dict[str, Dict[str, Any]] = {}
    groups: Optional[List[Dict[str, Any]]] = None
    for rank in range(world):
        path = folder / "optim" / f"rank{rank}.pt"
        if not path.is_file():
            raise OLMoCheckpointError(f"missing shard file {path}")
        shard = torch.load(path, map_location="cpu", weights_only=False)
        if groups is None:
            groups = shard["param_groups"]
        id_to_name = {pid: _clean(n) for g in shard["param_groups"] for n, pid in zip(g["param_names"], g["params"])}
        for pid, entries in shard["state"].items():
            name = id_to_name[pid] if pid in id_to_name else _clean(str(pid))
            piece = layout[rank].get(name)
            for key, value in entries.items():
                if not isinstance(value, torch.Tensor) or value.dim() == 0:
                    state.setdefault(name, {}).setdefault(key, value.to(dev) if isinstance(value, torch.Tensor) else value)
                    continue
                if value.numel() == 0:
                    continue
                if piece is None:
                    raise OLMoCheckpointError(f"optimizer state of {name} on rank {rank} has no matching parameter shard")
                if key not in state.setdefault(name, {}):
                    state[name][key] = torch.full(tuple(piece.shape), float("nan"), dtype=value.dtype, device=dev)
                piece.copy_into(state[name][key], value)
    assert groups is not None
    for g in groups:  # names instead of integer ids, so that the state can be scattered by name on restore
        g["param_names"] = [_clean(n) for n in g["param_names"]]
        g["params"] = list(g["param_names"])
    for name, entries in state.items():
        for key, value in entries.items():
            if isinstance(value, torch.Tensor) and value.dim() > 0 and torch.isnan(value).any():
                raise OLMoCheckpointError(f"optimizer state {key} of {name} was not fully covered by the shard files")
    return model_state, {"state": state, "param_groups": groups}, trainer_state


# --------------------------------------------------------------------------------------------- detection


def detect_layout(load_path: PathOrStr) -> str:
    """``flat_shard`` (this framework), ``torch_new``, ``torch_legacy``, ``local``, ``olmo_core`` or ``unsharded``."""
    folder = Path(load_path)
    if (folder / "model_and_optim" / ".metadata").is_file():
        return "torch_new"
    if (folder / "rank0.pt").is_file():
        return "torch_legacy"
    if (folder / "model.pt").is_file() or (folder / "model.safetensors").is_file():
        return "unsharded"
    meta_file = folder / "metadata.yaml"
    if meta_file.is_file():
        meta = yaml.safe_load(meta_file.read_text()) or {}
        if "format" in meta:
            return "flat_shard"
        if "world_size" in meta and (folder / "model" / "rank0.pt").is_file():
            return "local"
    if (folder / "model" / "metadata.json").is_file() or (folder / "model" / ".metadata").is_file() or (folder / "train" / "rank0.pt").is_file():
        return "olmo_core"
    raise OLMoCheckpointError(f"{folder} is not a checkpoint layout this framework knows")


def unshard_reference_checkpoint(
    load_path: PathOrStr, *, layout: Optional[str] = None, load_optimizer_state: bool = True, load_trainer_state: bool = True,
    device: Optional[torch.device] = None,
) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
    """Dispatch on the layout of a sharded checkpoint written by the reference implementation."""
    layout = layout or detect_layout(load_path)
    kw = dict(load_optimizer_state=load_optimizer_state, load_trainer_state=load_trainer_state)
    if layout == "torch_legacy":
        return unshard_torch_legacy_checkpoint(load_path, device=device, **kw)
    if layout == "local":
        return unshard_local_checkpoint(load_path, device=device, **kw)
    if layout == "torch_new":
        from .checkpoint import unshard_torch_dcp_checkpoint

        return unshard_torch_dcp_checkpoint(load_path, **kw)
    if layout == "olmo_core":
        raise OLMoCheckpointError(
            f"{load_path} looks like an olmo_core checkpoint; reading it needs the olmo_core package's own loader, which this "
            "framework does not bundle: unshard it with the tool that wrote it, then load the unsharded result here"
        )
    raise OLMoCheckpointError(f"{load_path}: layout '{layout}' is not a reference sharded layout")


# ------------------------------------------------------------------------------------------------ export


def export_torch_new_checkpoint(
    out_dir: PathOrStr, model_state: Dict[str, torch.Tensor], optim_state: Optional[Dict[str, Any]] = None,
    trainer_state: Optional[Dict[str, Any]] = None, *, world_size: int = 1,
) -> PathOrStr:
    """Write full states in the layout of the reference's ``torch_new`` sharded checkpointer
    (``olmo/checkpoint.py:99-144,892-966``): ``model_and_optim/`` in torch's distributed-checkpoint format holding
    ``model.<parameter>`` tensors, ``optim.state.<parameter>.<key>`` tensors and the parameter groups, plus
    ``train/rank{r}.pt``.  That format records every tensor as chunks with global offsets and is resharded by its
    reader, so one writer process produces a checkpoint that a job of any world size can load with FSDP's sharded state
    dicts; ``world_size`` only sets how many per-rank trainer-state files are written (each rank reads its own; 0: none,
    the caller writes them).
    ``optim_state`` is keyed by parameter name (``{"state": {name: {...}}, "param_groups": [{"params": [names], ...}]}``),
    the form of an unsharded ``optim.pt``."""
    import torch.distributed.checkpoint as dcp

    from .util import is_url, upload

    remote = is_url(str(out_dir))
    if remote:
        from .checkpoint import RemoteFileSystemWriter

        root = str(out_dir).rstrip("/")
        writer = RemoteFileSystemWriter(f"{root}/model_and_optim")
        out = root  # type: ignore[assignment]
    else:
        out = Path(out_dir)
        folder = out / "model_and_optim"
        folder.mkdir(parents=True, exist_ok=True)
        writer = dcp.FileSystemWriter(str(folder))
    payload: Dict[str, Any] = {"model": {name: t.detach().cpu().contiguous() for name, t in model_state.items()}}
    if optim_state is not None:
        groups = optim_state.get("param_groups", [])
        known = set(model_state)
        for group in groups:
            for name in group.get("params", []):
                if not isinstance(name, str) or name not in known:
                    raise OLMoCheckpointError(
                        f"parameter group entry {name!r} is not a parameter name of the model state; the export needs an "
                        "optimizer state keyed by parameter name"
                    )
        state = {
            name: {key: (v.detach().cpu().contiguous() if isinstance(v, torch.Tensor) else v) for key, v in entry.items()}
            for name, entry in optim_state.get("state", {}).items()
        }
        payload["optim"] = {"state": state, "param_groups": groups}
    dcp.save(payload, storage_writer=writer, no_dist=True)
    if world_size > 0 and remote:
        import tempfile

        with tempfile.TemporaryDirectory() as tmp:
            torch.save(trainer_state or {}, Path(tmp) / "train.pt")
            for rank in range(world_size):
                upload(Path(tmp) / "train.pt", f"{out}/train/rank{rank}.pt", save_overwrite=True)
    elif world_size > 0:
        (out / "train").mkdir(exist_ok=True)
        for rank in range(world_size):
            torch.save(trainer_state or {}, out / "train" / f"rank{rank}.pt")
    return out
