"""
Checkpointing (reference: ``olmo/checkpoint.py:99-2030``).

Two on-disk layouts:

*Unsharded* (``step{N}-unsharded/``) — byte-compatible with the reference: ``config.yaml``, ``model.pt``
(``{FQN: fp32 tensor}``), ``optim.pt`` (``{"state": {FQN: {...}}, "param_groups": [...]}``), ``train.pt``.  A sibling
``*.safetensors`` file is preferred on load.

*Sharded* (``step{N}/``) — this framework's flat-shard format.  Every rank writes the raw contents of its shards,

    model/rank{r}.pt   {"units": {unit name: fp32 master shard}}
    optim/rank{r}.pt   {"units": {unit name: {"exp_avg": shard, ...}}, "steps": {...}, "param_groups": [...]}
    train/rank{r}.pt   trainer state
    metadata.yaml      world/shard sizes and, per unit, the (FQN, shape, offset) table

so saving is one sequential write per rank with no gather, and restoring at the same world size is one read.  A
different world size, and :meth:`FlatShardCheckpointer.unshard_checkpoint`, reassemble full tensors from the shard
files through the metadata table.  All four ``sharded_checkpointer`` names of the reference select this format.

Writes go to ``{dir}-tmp`` and are renamed into place after a barrier, so an interrupted save never leaves a
directory that looks complete; ``config.yaml`` is written and uploaded last for the same reason.
"""
from __future__ import annotations

import io
import logging
import os
import pickle
import shutil
from abc import ABCMeta, abstractmethod
from concurrent.futures import ThreadPoolExecutor
from contextlib import contextmanager
from copy import deepcopy
from pathlib import Path
from typing import Any, Dict, Generator, List, Optional, Set, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import yaml

from .aliases import PathOrStr
from .config import ShardedCheckpointerType, TrainConfig
from .exceptions import OLMoCheckpointError
from .optim import Optimizer, fix_optim_state_dict
from .safetensors_util import safetensors_file_to_state_dict
from .torch_util import barrier, get_fs_local_rank, get_global_rank, get_world_size, is_distributed
from .util import default_thread_count, dir_is_empty, is_url, resource_path, upload, wait_for

__all__ = [
    "save_state_dict", "load_state_dict", "load_model_state", "Checkpointer", "FullCheckpointer",
    "FlatShardCheckpointer", "build_sharded_checkpointer", "TorchNewStyleShardedCheckpointer", "TorchLegacyShardedCheckpointer",
    "LocalShardedCheckpointer", "OlmoCoreCheckpointer", "RemoteFileSystemWriter", "RemoteFileSystemReader",
    "save_fsdp_model_and_optim_state", "load_fsdp_model_and_optim_state", "load_fsdp_optim_state", "unshard_torch_dcp_checkpoint", "is_torch_dcp_checkpoint",
]

log = logging.getLogger(__name__)

MODEL_AND_OPTIM_FOLDER = "model_and_optim"


# ------------------------------------------------------------------------------------- file helpers


def save_state_dict(
    checkpoint_dir: PathOrStr, fname: str, state_dict: Dict[str, Any], *, upload_to: Optional[str] = None,
    save_overwrite: bool = False, synchronize: bool = True,
) -> None:
    """``torch.save`` to ``checkpoint_dir/fname`` (sub-folders allowed), then optionally upload it."""
    target = Path(checkpoint_dir) / fname
    if save_overwrite:
        target.unlink(missing_ok=True)
    elif target.is_file():
        raise FileExistsError(target)
    if synchronize:
        barrier()
    target.parent.mkdir(exist_ok=True, parents=True)
    if synchronize:
        barrier()
    torch.save(state_dict, target)
    if upload_to is not None:
        dest = f"{upload_to.rstrip('/')}/{fname}"
        log.info("Uploading %s to %s...", target, dest)
        upload(target, dest, save_overwrite=save_overwrite)


def load_state_dict(checkpoint_dir: PathOrStr, fname: str, *, local_cache: Optional[PathOrStr] = None, map_location: Optional[str] = None):
    """Load ``fname`` from a local or remote checkpoint folder, preferring a ``.safetensors`` sibling."""
    if fname.endswith(".pt"):
        try:
            path = resource_path(str(checkpoint_dir).rstrip("/"), fname[:-3] + ".safetensors", local_cache=local_cache)
            return safetensors_file_to_state_dict(path, map_location=map_location)
        except FileNotFoundError:
            pass
    path = resource_path(str(checkpoint_dir).rstrip("/"), fname, local_cache=local_cache)
    try:
        if str(map_location) == "cpu":
            # Map the file instead of reading it: the ranks of a node that restore from the same file then share its pages
            # through the page cache instead of each holding a private copy (the mapping is private: writes to the tensors
            # never reach the file).  Files in torch's older, non-archive format cannot be mapped and are read.
            try:
                return torch.load(path, map_location=map_location, weights_only=False, mmap=True)
            except (RuntimeError, ValueError) as e:
                if "mmap" not in str(e):
                    raise
        return torch.load(path, map_location=map_location, weights_only=False)
    except (RuntimeError, EOFError, pickle.UnpicklingError, ValueError, OSError) as e:
        if isinstance(e, FileNotFoundError):
            raise
        # a file cut short by a crash or a failed transfer must stop the restore with the file's name, not surface as an
        # archive-format error from deep inside the loader
        raise OLMoCheckpointError(f"{path} is truncated or corrupt ({type(e).__name__}: {str(e)[:200]})") from e


def _engine_of(dist_model: nn.Module):
    return getattr(dist_model, "engine", None)


def _plain_module(dist_model: nn.Module) -> nn.Module:
    return getattr(dist_model, "module", dist_model)


def _clean_param_groups(optim: Optimizer) -> List[Dict[str, Any]]:
    groups = []
    for g in optim.state_dict()["param_groups"]:
        g = dict(g)
        g["params"] = list(g["param_names"])
        groups.append(g)
    return groups


def load_model_state(checkpoint_dir: PathOrStr, model: nn.Module) -> None:
    """Load only the weights of a sharded checkpoint into an unwrapped model."""
    state, _, _ = FlatShardCheckpointer(TrainConfig()).unshard_checkpoint(checkpoint_dir, load_optimizer_state=False, load_trainer_state=False)
    model.load_state_dict(model._make_state_dict_compatible(state)[0] if hasattr(model, "_make_state_dict_compatible") else state)


# ------------------------------------------------------------------------------------- base class


class Checkpointer(metaclass=ABCMeta):
    def __init__(self, cfg: TrainConfig, thread_count: Optional[int] = None):
        self.cfg = cfg
        self.thread_count = thread_count or default_thread_count()

    @abstractmethod
    def save_checkpoint(self, dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, train_state: Dict[str, Any], *, upload_to: Optional[str] = None) -> None:
        raise NotImplementedError

    @abstractmethod
    def restore_checkpoint(
        self, load_path: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, local_cache: Optional[PathOrStr] = None,
        load_optimizer_state: bool = True,
    ) -> Dict[str, Any]:
        """Restore model (and optimizer) in place; return the trainer state."""
        raise NotImplementedError

    def unshard_checkpoint(
        self, load_path: PathOrStr, *, local_cache: Optional[PathOrStr] = None, load_optimizer_state: bool = True,
        load_trainer_state: bool = True, device: Optional[torch.device] = None,
    ) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
        raise NotImplementedError

    @contextmanager
    def _temporary_wd(self, dir: PathOrStr) -> Generator[Path, None, None]:
        """Yield ``{dir}-tmp``; on normal exit rename it to ``dir``.  Filesystem-local rank 0 creates and renames,
        everyone waits until the result is visible (shared filesystems can lag)."""
        final = Path(dir)
        if not dir_is_empty(final):
            if not self.cfg.save_overwrite:
                raise FileExistsError(final)
            if get_fs_local_rank() == 0:
                shutil.rmtree(final, ignore_errors=True)
        barrier()
        tmp = final.with_name(final.name + "-tmp")
        if get_fs_local_rank() == 0:
            shutil.rmtree(tmp, ignore_errors=True)
            tmp.mkdir(exist_ok=True, parents=True)
        wait_for(lambda: tmp.exists(), "Waiting for checkpoint directory", timeout=10.0)
        barrier()
        yield tmp
        barrier()
        if get_fs_local_rank() == 0:
            try:
                tmp.replace(final)
            except FileNotFoundError:
                if not final.exists():  # another filesystem-local rank 0 on a shared disk already renamed it
                    raise
        wait_for(lambda: final.exists(), "Waiting for checkpoint directory", timeout=10.0)
        barrier()

    def _save_config(self, dir: PathOrStr, *, upload_to: Optional[str] = None) -> None:
        if get_global_rank() == 0:
            log.info("Saving config...")
            path = Path(dir) / "config.yaml"
            self.cfg.save(path)
            if upload_to is not None:
                upload(path, f"{upload_to}/config.yaml", save_overwrite=self.cfg.save_overwrite)


# ---------------------------------------------------------------------------------- unsharded format


def _optim_state_by_name(optim: Optimizer) -> Dict[str, Dict[str, Any]]:
    out = {}
    for group in optim.param_groups:
        for name, p in zip(group["param_names"], group["params"]):
            out[name] = optim.state.get(p, {})
    return out


class FullCheckpointer(Checkpointer):
    """Whole tensors gathered to rank 0 (``model.pt``, ``optim.pt``, ``train.pt``, ``config.yaml``)."""

    # -- gather
    def _full_model_state(self, dist_model: nn.Module) -> Dict[str, torch.Tensor]:
        engine = _engine_of(dist_model)
        if engine is not None:
            return engine.full_model_state_dict(rank0_only=True, cpu=True)
        return {k: v.detach().float().cpu() for k, v in _plain_module(dist_model).state_dict().items()}

    def _full_optim_state(self, dist_model: nn.Module, optim: Optimizer) -> Dict[str, Any]:
        engine = _engine_of(dist_model)
        by_name = _optim_state_by_name(optim)
        state: Dict[str, Dict[str, Any]] = {}
        if engine is None or not engine.is_sharded:
            for name, st in by_name.items():
                if st:
                    state[name] = {k: (v.detach().cpu().clone() if isinstance(v, torch.Tensor) else v) for k, v in st.items()}
        else:
            keep = get_global_rank() == 0
            # Scalar entries (``step``, running gradient norms) and the set of tensor keys are collected from every rank:
            # a rank whose shard of a parameter is empty may hold no state for it at all, and rank 0 is such a rank for
            # the parameters at the end of every unit.
            local_scalars: Dict[str, Dict[str, Tuple[bool, Any]]] = {}
            for name, st in by_name.items():
                for k, v in st.items():
                    if isinstance(v, torch.Tensor) and v.dim() > 0:
                        continue
                    local_scalars.setdefault(name, {})[k] = (True, float(v.item())) if isinstance(v, torch.Tensor) else (False, v)
            local_keys = sorted({k for st in by_name.values() for k, v in st.items() if isinstance(v, torch.Tensor) and v.dim() > 0})
            every: List[Any] = [None] * get_world_size()
            if is_distributed():
                dist.all_gather_object(every, (local_keys, local_scalars))
            else:
                every = [(local_keys, local_scalars)]
            tensor_keys = sorted({k for keys, _ in every for k in keys})
            for unit in engine.units:
                lo = engine.shard_rank * unit.shard_size
                for key in tensor_keys:
                    shard = torch.zeros(unit.shard_size, dtype=torch.float32, device=engine.device)
                    for s in unit.slots:
                        st = by_name.get(s.name, {})
                        if key in st and st[key].numel() > 0:
                            a = max(s.offset, lo) - lo
                            shard[a : a + st[key].numel()].copy_(st[key].reshape(-1))
                    full = engine.full_tensor(unit, shard)
                    if keep:
                        # every slot gets the key; slots that never received state on any rank are dropped below
                        for s in unit.slots:
                            state.setdefault(s.name, {})[key] = full[s.offset : s.offset + s.numel].view(s.shape).cpu().clone()
                    del full, shard
            if keep:
                for _, scalars in every:
                    for name, entries in scalars.items():
                        cur = state.setdefault(name, {})
                        for k, (was_tensor, v) in entries.items():
                            if k == "step" and k in cur:  # ranks that skipped empty shards lag behind: the furthest count is the true one
                                v = max(v, float(cur[k]))
                            elif k in cur:
                                continue
                            cur[k] = torch.tensor(v, dtype=torch.float32) if was_tensor else v
                # drop entries of parameters that never received state on any rank
                state = {n: s for n, s in state.items() if "step" in s or not tensor_keys}
        return {"state": state, "param_groups": _clean_param_groups(optim)}

    def save_checkpoint(self, dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, trainer_state: Dict[str, Any], *, upload_to: Optional[str] = None) -> None:
        with self._temporary_wd(dir) as tmp:
            model_state = self._full_model_state(dist_model)
            if get_global_rank() == 0:
                log.info("Saving model state...")
                save_state_dict(tmp, "model.pt", model_state, upload_to=upload_to, save_overwrite=self.cfg.save_overwrite, synchronize=False)
            del model_state
            barrier()
            optim_state = self._full_optim_state(dist_model, optim)
            if get_global_rank() == 0:
                log.info("Saving optim state...")
                save_state_dict(tmp, "optim.pt", optim_state, upload_to=upload_to, save_overwrite=self.cfg.save_overwrite, synchronize=False)
                log.info("Saving trainer state...")
                save_state_dict(tmp, "train.pt", trainer_state, upload_to=upload_to, save_overwrite=self.cfg.save_overwrite, synchronize=False)
            del optim_state
            barrier()
            self._save_config(tmp, upload_to=upload_to)

    # -- restore
    @staticmethod
    def _normalise_optim_state(optim_state: Dict[str, Any], renames: Dict[str, Set[str]]) -> Dict[str, Any]:
        """Key the optimizer state by clean FQN (it may arrive keyed by integer ids) and follow model-key renames."""
        groups = optim_state["param_groups"]
        if groups and groups[0]["params"] and isinstance(groups[0]["params"][0], int):
            id_to_name = {}
            for g in groups:
                names = [n.replace("_fsdp_wrapped_module.", "") for n in g["param_names"]]
                id_to_name.update(dict(zip(g["params"], names)))
                g["param_names"] = g["params"] = names
            optim_state["state"] = {id_to_name[i]: s for i, s in optim_state["state"].items()}
        else:
            for g in groups:
                g["param_names"] = g["params"] = [n.replace("_fsdp_wrapped_module.", "") for n in g.get("param_names", g["params"])]
            optim_state["state"] = {k.replace("_fsdp_wrapped_module.", ""): s for k, s in optim_state["state"].items()}
        for old, news in renames.items():
            if old in news and len(news) == 1:
                continue
            st = optim_state["state"].pop(old, None)
            if st is not None:
                for i, new in enumerate(sorted(news)):
                    optim_state["state"][new] = st if i == 0 else deepcopy(st)
        for g in groups:
            g["params"] = g["param_names"] = [new for old in g["params"] for new in sorted(renames.get(old, {old}))]
        return optim_state

    @staticmethod
    def load_optim_state_into(dist_model: nn.Module, optim: Optimizer, optim_state: Dict[str, Any]) -> None:
        """Scatter a full, FQN-keyed optimizer state into the live optimizer (each rank keeps its shard ranges)."""
        engine = _engine_of(dist_model)
        ranges = engine.param_shard_ranges() if engine is not None else {}
        optim_state = fix_optim_state_dict(optim, optim_state)
        for group, saved in zip(optim.param_groups, optim_state["param_groups"]):
            for k, v in saved.items():
                if k not in ("params", "param_names"):
                    group[k] = v
        for group in optim.param_groups:
            for name, p in zip(group["param_names"], group["params"]):
                saved = optim_state["state"].get(name)
                if not saved:
                    continue
                st = optim.state[p]
                for key, value in saved.items():
                    if isinstance(value, torch.Tensor) and value.dim() > 0:
                        a, b, _ = ranges.get(name, (0, value.numel(), value.numel()))
                        piece = value.reshape(-1)[a:b].to(p.device, torch.float32).view(p.shape)
                        if key in st and isinstance(st[key], torch.Tensor) and st[key].shape == piece.shape:
                            st[key].copy_(piece)
                        else:
                            st[key] = piece.clone()
                    else:
                        st[key] = value.clone().float().cpu() if isinstance(value, torch.Tensor) else value

    def restore_checkpoint(
        self, load_path: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, local_cache: Optional[PathOrStr] = None,
        load_optimizer_state: bool = True,
    ) -> Dict[str, Any]:
        module = _plain_module(dist_model)
        engine = _engine_of(dist_model)
        model_state = load_state_dict(load_path, "model.pt", local_cache=local_cache, map_location="cpu")
        renames: Dict[str, Set[str]] = {}
        if hasattr(module, "_make_state_dict_compatible"):
            model_state, renames = module._make_state_dict_compatible(model_state)
        if engine is not None:
            engine.load_full_model_state_dict(model_state)
        else:
            module.load_state_dict(model_state)
        del model_state
        if load_optimizer_state:
            optim_state = load_state_dict(load_path, "optim.pt", local_cache=local_cache, map_location="cpu")
            optim_state = self._normalise_optim_state(optim_state, renames)
            self.load_optim_state_into(dist_model, optim, optim_state)
            del optim_state
        try:
            trainer_state = load_state_dict(load_path, "train.pt", local_cache=local_cache)
        except FileNotFoundError:
            trainer_state = load_state_dict(load_path, "other.pt", local_cache=local_cache)  # pre-0.3 name
        barrier()
        return trainer_state

    def load_checkpoint(
        self, load_path: PathOrStr, *, local_cache: Optional[PathOrStr] = None, load_optimizer_state: bool = True,
        device: Optional[torch.device] = None,
    ) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]]]:
        dev = str(device) if device is not None else "cpu"
        model_state = load_state_dict(load_path, "model.pt", local_cache=local_cache, map_location=dev)
        optim_state = load_state_dict(load_path, "optim.pt", local_cache=local_cache, map_location=dev) if load_optimizer_state else None
        return model_state, optim_state


# ------------------------------------------------------------------------------------ sharded format


class FlatShardCheckpointer(Checkpointer):
    """Per-rank raw shard files plus a layout table (see the module docstring)."""

    format_name = "flat_shard_v1"

    def _layout(self, engine) -> Dict[str, Any]:
        return {
            "format": self.format_name,
            "world_size": get_world_size(),
            "shard_world": engine.shard_world,
            "num_replicas": engine.num_replicas,
            "units": [
                {
                    "name": u.name, "numel": u.numel, "shard_size": u.shard_size,
                    "params": [{"name": s.name, "shape": list(s.shape), "offset": s.offset} for s in u.slots],
                }
                for u in engine.units
            ],
        }

    def save_checkpoint(self, dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, trainer_state: Dict[str, Any], *, upload_to: Optional[str] = None) -> None:
        engine = _engine_of(dist_model)
        if engine is None:
            raise OLMoCheckpointError("sharded checkpoints need a flat-shard engine; use an unsharded checkpoint instead")
        rank = get_global_rank()
        with self._temporary_wd(dir) as tmp:
            # replicas hold identical shards; only the first replica writes model/optim files
            writes_shards = rank < engine.shard_world
            if writes_shards:
                save_state_dict(
                    tmp, f"model/rank{engine.shard_rank}.pt", {"units": {u.name: u.master.detach().cpu() for u in engine.units}},
                    upload_to=upload_to, save_overwrite=self.cfg.save_overwrite, synchronize=False,
                )
                by_name = _optim_state_by_name(optim)
                units_state: Dict[str, Dict[str, torch.Tensor]] = {}
                scalars: Dict[str, Dict[str, Any]] = {}
                for u in engine.units:
                    lo = engine.shard_rank * u.shard_size
                    per_key: Dict[str, torch.Tensor] = {}
                    for s in u.slots:
                        for key, value in by_name.get(s.name, {}).items():
                            if isinstance(value, torch.Tensor) and value.dim() > 0:
                                buf = per_key.setdefault(key, torch.zeros(u.shard_size, dtype=torch.float32))
                                a = max(s.offset, lo) - lo
                                buf[a : a + value.numel()].copy_(value.reshape(-1))
                            else:
                                scalars.setdefault(s.name, {})[key] = value.detach().cpu() if isinstance(value, torch.Tensor) else value
                    units_state[u.name] = per_key
                save_state_dict(
                    tmp, f"optim/rank{engine.shard_rank}.pt",
                    {"units": units_state, "scalars": scalars, "param_groups": _clean_param_groups(optim)},
                    upload_to=upload_to, save_overwrite=self.cfg.save_overwrite, synchronize=False,
                )
            save_state_dict(tmp, f"train/rank{rank}.pt", trainer_state, upload_to=upload_to, save_overwrite=self.cfg.save_overwrite, synchronize=False)
            if rank == 0:
                meta = tmp / "metadata.yaml"
                meta.write_text(yaml.safe_dump(self._layout(engine), sort_keys=False))
                if upload_to is not None:
                    upload(meta, f"{upload_to}/metadata.yaml", save_overwrite=self.cfg.save_overwrite)
            barrier()
            self._save_config(tmp, upload_to=upload_to)

    @staticmethod
    def _read_meta(load_path: PathOrStr, local_cache: Optional[PathOrStr]) -> Dict[str, Any]:
        meta = yaml.safe_load(resource_path(str(load_path).rstrip("/"), "metadata.yaml", local_cache=local_cache).read_text())
        if meta.get("format") != FlatShardCheckpointer.format_name:
            raise OLMoCheckpointError(f"{load_path} is not a flat-shard checkpoint (format={meta.get('format')})")
        return meta

    def restore_checkpoint(
        self, load_path: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, local_cache: Optional[PathOrStr] = None,
        load_optimizer_state: bool = True,
    ) -> Dict[str, Any]:
        engine = _engine_of(dist_model)
        if engine is None:
            raise OLMoCheckpointError("restoring a sharded checkpoint needs a flat-shard engine")
        foreign = self._foreign_layout(load_path)
        if foreign is not None:
            return self._restore_foreign(load_path, foreign, dist_model, optim, load_optimizer_state=load_optimizer_state)
        meta = self._read_meta(load_path, local_cache)
        # raw shards may only be copied when the whole layout agrees: unit order and sizes, and every parameter's name,
        # shape and offset inside its unit (equal sizes alone would let a changed wrapping put shards into the wrong slots)
        mine = self._layout(engine)
        same_layout = meta["shard_world"] == mine["shard_world"] and [
            (u["name"], u["numel"], [(p["name"], list(p["shape"]), p["offset"]) for p in u["params"]]) for u in meta["units"]
        ] == [(u["name"], u["numel"], [(p["name"], list(p["shape"]), p["offset"]) for p in u["params"]]) for u in mine["units"]]
        if same_layout:
            shard = load_state_dict(load_path, f"model/rank{engine.shard_rank}.pt", local_cache=local_cache, map_location="cpu")
            for u in engine.units:
                src = shard["units"][u.name]
                if not torch.isfinite(src).all():
                    raise OLMoCheckpointError(f"non-finite values in shard of unit {u.name}")
                u.master.copy_(src)
                u.lowp.copy_(src) if u.lowp.data_ptr() != u.master.data_ptr() else None
            engine._params_stale = True
            if getattr(engine, "comm", None) is not None:
                engine.params_changed()  # peers gather from these shards: open a new parameter epoch once all ranks are done
            if not engine.is_sharded:
                for u in engine.units:
                    if u.full.data_ptr() != u.master.data_ptr():
                        u.full.copy_(u.master)
                engine._params_stale = False
            if load_optimizer_state:
                saved = load_state_dict(load_path, f"optim/rank{engine.shard_rank}.pt", local_cache=local_cache, map_location="cpu")
                self._load_optim_shards(engine, optim, saved)
        else:
            log.info("Checkpoint layout differs from the running job (saved shard world %d); resharding", meta["shard_world"])
            model_state, optim_state, _ = self.unshard_checkpoint(load_path, local_cache=local_cache, load_optimizer_state=load_optimizer_state, load_trainer_state=False)
            engine.load_full_model_state_dict(model_state)
            if load_optimizer_state and optim_state is not None:
                FullCheckpointer.load_optim_state_into(dist_model, optim, optim_state)
        rank = get_global_rank()
        try:
            trainer_state = load_state_dict(load_path, f"train/rank{rank}.pt", local_cache=local_cache)
        except FileNotFoundError:
            trainer_state = load_state_dict(load_path, "train/rank0.pt", local_cache=local_cache)  # world size changed
        barrier()
        return trainer_state

    @staticmethod
    def _foreign_layout(load_path: PathOrStr) -> Optional[str]:
        """Name of the reference layout found at ``load_path`` (local directories only), or ``None`` for this framework's own."""
        if is_url(load_path):
            return None
        from .checkpoint_compat import detect_layout

        try:
            layout = detect_layout(load_path)
        except OLMoCheckpointError:
            return None
        return layout if layout in ("torch_new", "torch_legacy", "local", "olmo_core") else None

    def _restore_foreign(self, load_path: PathOrStr, layout: str, dist_model: nn.Module, optim: Optimizer, *, load_optimizer_state: bool) -> Dict[str, Any]:
        """Resume from a sharded checkpoint the reference wrote: every rank reassembles the full tensors on the host and
        keeps its own ranges (the writing job's world size does not have to match)."""
        from .checkpoint_compat import unshard_reference_checkpoint

        log.info("%s is a '%s' checkpoint of the reference implementation; unsharding it on the host", load_path, layout)
        engine = _engine_of(dist_model)
        model_state, optim_state, trainer_state = unshard_reference_checkpoint(
            load_path, layout=layout, load_optimizer_state=load_optimizer_state, load_trainer_state=True
        )
        engine.load_full_model_state_dict(model_state)
        del model_state
        if load_optimizer_state and optim_state is not None:
            optim_state = FullCheckpointer._normalise_optim_state(optim_state, {})
            FullCheckpointer.load_optim_state_into(dist_model, optim, optim_state)
        barrier()
        return trainer_state or {}

    @staticmethod
    def _load_optim_shards(engine, optim: Optimizer, saved: Dict[str, Any]) -> None:
        saved = fix_optim_state_dict(optim, saved)
        for group, sg in zip(optim.param_groups, saved["param_groups"]):
            for k, v in sg.items():
                if k not in ("params", "param_names"):
                    group[k] = v
        by_name = {name: p for g in optim.param_groups for name, p in zip(g["param_names"], g["params"])}
        for u in engine.units:
            lo = engine.shard_rank * u.shard_size
            for key, buf in saved["units"].get(u.name, {}).items():
                for s in u.slots:
                    p = by_name.get(s.name)
                    if p is None or p.numel() == 0:
                        continue
                    a = max(s.offset, lo) - lo
                    piece = buf[a : a + p.numel()].to(p.device).view(p.shape)
                    st = optim.state[p]
                    if key in st and isinstance(st[key], torch.Tensor) and st[key].shape == piece.shape:
                        st[key].copy_(piece)
                    else:
                        st[key] = piece.clone()
        for name, sc in saved.get("scalars", {}).items():
            p = by_name.get(name)
            if p is not None:
                for k, v in sc.items():
                    optim.state[p][k] = v.clone() if isinstance(v, torch.Tensor) else v

    def unshard_checkpoint(
        self, load_path: PathOrStr, *, local_cache: Optional[PathOrStr] = None, load_optimizer_state: bool = True,
        load_trainer_state: bool = True, device: Optional[torch.device] = None,
    ) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
        """Reassemble full tensors offline (no process group needed): shard files are read by a thread pool, full
        buffers start as NaN and are verified finite after the copy so a missing shard cannot go unnoticed."""
        foreign = self._foreign_layout(load_path)
        if foreign is not None:
            from .checkpoint_compat import unshard_reference_checkpoint

            return unshard_reference_checkpoint(
                load_path, layout=foreign, load_optimizer_state=load_optimizer_state, load_trainer_state=load_trainer_state, device=device
            )
        meta = self._read_meta(load_path, local_cache)
        sw = meta["shard_world"]
        dev = "cpu" if device is None else str(device)

        def read(kind: str, r: int):
            return load_state_dict(load_path, f"{kind}/rank{r}.pt", local_cache=local_cache, map_location="cpu")

        with ThreadPoolExecutor(max_workers=self.thread_count) as pool:
            model_shards = list(pool.map(lambda r: read("model", r), range(sw)))
            optim_shards = list(pool.map(lambda r: read("optim", r), range(sw))) if load_optimizer_state else None

        def assemble(per_rank: List[torch.Tensor], unit: Dict[str, Any]) -> torch.Tensor:
            full = torch.full((unit["numel"],), float("nan"), dtype=torch.float32)
            for r, piece in enumerate(per_rank):
                full[r * unit["shard_size"] : (r + 1) * unit["shard_size"]].copy_(piece)
            return full

        model_state: Dict[str, torch.Tensor] = {}
        for unit in meta["units"]:
            full = assemble([ms["units"][unit["name"]] for ms in model_shards], unit)
            for p in unit["params"]:
                n = 1
                for d in p["shape"]:
                    n *= d
                t = full[p["offset"] : p["offset"] + n].view(p["shape"]).clone()
                if not torch.isfinite(t).all():
                    raise OLMoCheckpointError(f"parameter {p['name']} was not fully covered by the shard files")
                model_state[p["name"]] = t.to(dev)
        optim_state: Optional[Dict[str, Any]] = None
        if optim_shards is not None:
            state: Dict[str, Dict[str, Any]] = {}
            for unit in meta["units"]:
                keys = sorted({k for os_ in optim_shards for k in os_["units"].get(unit["name"], {})})
                for key in keys:
                    full = assemble([os_["units"][unit["name"]].get(key, torch.zeros(unit["shard_size"])) for os_ in optim_shards], unit)
                    for p in unit["params"]:
                        n = 1
                        for d in p["shape"]:
                            n *= d
                        state.setdefault(p["name"], {})[key] = full[p["offset"] : p["offset"] + n].view(p["shape"]).clone().to(dev)
            for os_ in optim_shards:
                for name, sc in os_.get("scalars", {}).items():
                    for k, v in sc.items():
                        state.setdefault(name, {}).setdefault(k, v)
            optim_state = {"state": state, "param_groups": optim_shards[0]["param_groups"]}
        trainer_state = load_state_dict(load_path, "train/rank0.pt", local_cache=local_cache) if load_trainer_state else None
        return model_state, optim_state, trainer_state


def is_torch_dcp_checkpoint(load_path: PathOrStr) -> bool:
    """True for the layout the reference's ``torch_new`` sharded checkpointer writes: a ``model_and_optim/`` folder
    in ``torch.distributed.checkpoint`` format (``olmo/checkpoint.py:99-144``, ``:892-966``)."""
    if is_url(load_path):
        return False
    return (Path(load_path) / "model_and_optim" / ".metadata").is_file()


def unshard_torch_dcp_checkpoint(
    load_path: PathOrStr, *, load_optimizer_state: bool = True, load_trainer_state: bool = True
) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
    """Read a sharded checkpoint written by the reference's ``torch_new`` checkpointer (model and optimizer as FSDP
    sharded state dicts under ``model_and_optim/``, trainer state under ``train/rank*.pt``) into full tensors, in one
    CPU process.  The chunk layout is whatever the writing job's world size produced; the checkpoint library's reader
    reassembles whole tensors from the chunk table, so no process group is needed.  Optimizer state comes back keyed
    by parameter name, which ``FullCheckpointer`` accepts on restore."""
    from torch.distributed.checkpoint import FileSystemReader
    from torch.distributed.checkpoint.metadata import BytesStorageMetadata, TensorStorageMetadata
    from torch.distributed.checkpoint.state_dict_loader import _load_state_dict

    if is_url(str(load_path)):
        reader = RemoteFileSystemReader(f"{str(load_path).rstrip('/')}/model_and_optim")
        folder = f"{str(load_path).rstrip('/')}/model_and_optim"
    else:
        folder = Path(load_path) / "model_and_optim"
        reader = FileSystemReader(str(folder))
    table = reader.read_metadata().state_dict_metadata
    wanted: Dict[str, Any] = {}
    for key, entry in table.items():
        if not (key.startswith("model.") or load_optimizer_state):
            continue
        if isinstance(entry, TensorStorageMetadata):
            wanted[key] = torch.empty(entry.size, dtype=entry.properties.dtype)
        elif isinstance(entry, BytesStorageMetadata):
            wanted[key] = io.BytesIO()  # replaced by the unpickled object on load
    _load_state_dict(wanted, storage_reader=reader, no_dist=True)

    model_state: Dict[str, torch.Tensor] = {}
    optim_state: Optional[Dict[str, Any]] = {"state": {}, "param_groups": []} if load_optimizer_state else None
    flat_groups: Dict[int, Dict[str, Any]] = {}
    for key, value in wanted.items():
        if key.startswith("model."):
            model_state[key[len("model.") :].replace("_fsdp_wrapped_module.", "")] = value
        elif optim_state is not None and key.startswith("optim.state."):
            # "optim.state.<parameter name>.<state key>": the state key has no dot, the parameter name does
            name, _, state_key = key[len("optim.state.") :].rpartition(".")
            optim_state["state"].setdefault(name.replace("_fsdp_wrapped_module.", ""), {})[state_key] = value
        elif optim_state is not None and key == "optim.param_groups":  # stored as one pickled list
            optim_state["param_groups"] = value
        elif optim_state is not None and key.startswith("optim.param_groups."):  # or one entry per group and field
            index, _, field_name = key[len("optim.param_groups.") :].partition(".")
            flat_groups.setdefault(int(index), {})[field_name] = value
    if not model_state:
        raise OLMoCheckpointError(f"no model tensors found in {folder}")
    if optim_state is not None and flat_groups:
        optim_state["param_groups"] = [flat_groups[i] for i in sorted(flat_groups)]
    if optim_state is not None:
        for group in optim_state["param_groups"]:
            if isinstance(group, dict) and "params" in group:
                group["params"] = [str(n).replace("_fsdp_wrapped_module.", "") for n in group["params"]]

    trainer_state = None
    if load_trainer_state:
        for candidate in ("train/rank0.pt", "train.pt"):
            try:
                trainer_state = load_state_dict(load_path, candidate, map_location="cpu")
                break
            except FileNotFoundError:
                continue
    return model_state, optim_state, trainer_state


# ------------------------------------------------------------- torch distributed-checkpoint files on remote storage


class _RangeReader(io.RawIOBase):
    """A seekable read-only view of one remote object that fetches byte ranges on demand."""

    def __init__(self, url: str):
        super().__init__()
        from .util import file_size

        self.url, self.size, self.pos = url, file_size(url), 0

    def readable(self) -> bool:
        return True

    def seekable(self) -> bool:
        return True

    def tell(self) -> int:
        return self.pos

    def seek(self, offset: int, whence: int = io.SEEK_SET) -> int:
        base = {io.SEEK_SET: 0, io.SEEK_CUR: self.pos, io.SEEK_END: self.size}[whence]
        self.pos = max(0, min(self.size, base + offset))
        return self.pos

    def readinto(self, buffer) -> int:
        from .util import get_bytes_range

        want = min(len(buffer), self.size - self.pos)
        if want <= 0:
            return 0
        data = get_bytes_range(self.url, self.pos, want)
        buffer[: len(data)] = data
        self.pos += len(data)
        return len(data)


def _remote_file_system():
    """torch's checkpoint file-system interface over this framework's storage layer (any registered URL scheme).
    Writes go to a local temporary file that is uploaded when the stream closes; reads fetch byte ranges on demand."""
    import tempfile

    from torch.distributed.checkpoint.filesystem import FileSystemBase

    from .util import delete_file, file_size

    class RemoteFileSystem(FileSystemBase):
        @contextmanager
        def create_stream(self, path, mode: str):
            url = str(path)
            if mode == "rb":
                stream = io.BufferedReader(_RangeReader(url), buffer_size=8 << 20)
                try:
                    yield stream
                finally:
                    stream.close()
            elif mode == "wb":
                fd, tmp = tempfile.mkstemp(suffix=".distcp")
                try:
                    with os.fdopen(fd, "wb") as f:
                        yield f
                    upload(Path(tmp), url, save_overwrite=True)
                finally:
                    Path(tmp).unlink(missing_ok=True)
            else:
                raise ValueError(f"unsupported mode {mode!r}")

        def concat_path(self, path, suffix: str) -> str:
            return f"{str(path).rstrip('/')}/{suffix}"

        def init_path(self, path) -> str:
            return str(path)

        def rename(self, path, new_path) -> None:  # object stores have no rename: copy, then remove the source
            with self.create_stream(path, "rb") as src, self.create_stream(new_path, "wb") as dst:
                shutil.copyfileobj(src, dst, length=8 << 20)
            delete_file(str(path))

        def mkdir(self, path) -> None:
            pass  # prefixes need no creation

        @classmethod
        def validate_checkpoint_id(cls, checkpoint_id) -> bool:
            return is_url(str(checkpoint_id))

        def exists(self, path) -> bool:
            try:
                file_size(str(path))
                return True
            except FileNotFoundError:
                return False

        def rm_file(self, path) -> None:
            delete_file(str(path))

    return RemoteFileSystem()


def RemoteFileSystemWriter(path: PathOrStr, **kwargs):
    """A ``torch.distributed.checkpoint`` storage writer whose destination is a URL (the reference's class of this name,
    ``olmo/checkpoint.py:219-372``, writes locally and uploads per file as well).  Returns a ``FileSystemWriter`` bound to
    the remote file system."""
    from torch.distributed.checkpoint import FileSystemWriter

    kwargs.setdefault("sync_files", False)
    writer = FileSystemWriter(tempfile_safe_path(), **kwargs)
    writer.fs = _remote_file_system()
    writer.path = writer.fs.init_path(str(path))
    return writer


def RemoteFileSystemReader(path: PathOrStr, **kwargs):
    """The matching storage reader: reads ``.metadata`` and the data files of a checkpoint under a URL by byte range
    (``olmo/checkpoint.py:375-474``)."""
    from torch.distributed.checkpoint import FileSystemReader

    reader = FileSystemReader(tempfile_safe_path(), **kwargs)
    reader.fs = _remote_file_system()
    reader.path = reader.fs.init_path(str(path))
    return reader


def tempfile_safe_path() -> str:
    """A local path handed to the base classes' constructors (they normalise it as a local path; it is replaced at once)."""
    import tempfile

    return tempfile.gettempdir()


# ------------------------------------------------------------------ the reference's ``torch_new`` layout, live


def save_fsdp_model_and_optim_state(
    checkpoint_dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, upload_to: Optional[str] = None, save_overwrite: bool = False,
) -> None:
    """Write ``checkpoint_dir/model_and_optim/`` in the layout of the reference's function of the same name
    (``olmo/checkpoint.py:99-144``): torch's distributed-checkpoint format with ``model.<name>`` and
    ``optim.state.<name>.<key>`` entries.  The full tensors are gathered to rank 0, which writes them (the format stores
    global offsets and is resharded on load, so the writer's world size is not part of it)."""
    from .checkpoint_compat import export_torch_new_checkpoint

    target = Path(checkpoint_dir) / MODEL_AND_OPTIM_FOLDER
    if get_fs_local_rank() == 0 and target.is_dir() and any(target.iterdir()):
        if not save_overwrite:
            raise FileExistsError(target)
        shutil.rmtree(target, ignore_errors=True)
    barrier()
    gatherer = FullCheckpointer(None)  # type: ignore[arg-type]  # only its gather helpers are used; they read no settings
    model_state = gatherer._full_model_state(dist_model)
    optim_state = gatherer._full_optim_state(dist_model, optim)
    if get_global_rank() == 0:
        export_torch_new_checkpoint(checkpoint_dir, model_state, optim_state, None, world_size=0)
        if upload_to is not None:
            for path in sorted(target.rglob("*")):
                if path.is_file():
                    upload(path, f"{upload_to.rstrip('/')}/{MODEL_AND_OPTIM_FOLDER}/{path.relative_to(target)}", save_overwrite=save_overwrite)
    del model_state, optim_state
    barrier()


def load_fsdp_model_and_optim_state(
    checkpoint_dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, local_cache: Optional[PathOrStr] = None,
    load_optimizer_state: bool = True,
) -> None:
    """Restore model (and optimizer) in place from a ``model_and_optim/`` folder in the reference's ``torch_new`` layout,
    whoever wrote it and at whatever world size (``olmo/checkpoint.py:147-216``)."""
    source = local_cache if local_cache is not None and is_torch_dcp_checkpoint(local_cache) else checkpoint_dir
    model_state, optim_state, _ = unshard_torch_dcp_checkpoint(source, load_optimizer_state=load_optimizer_state, load_trainer_state=False)
    engine = _engine_of(dist_model)
    if engine is not None:
        engine.load_full_model_state_dict(model_state)
    else:
        _plain_module(dist_model).load_state_dict(model_state)
    if load_optimizer_state and optim_state is not None:
        FullCheckpointer.load_optim_state_into(dist_model, optim, FullCheckpointer._normalise_optim_state(optim_state, {}))
    barrier()


def load_fsdp_optim_state(dist_model: nn.Module, optim: Optimizer, optim_state: Dict[str, Any]) -> None:
    """Load a *full* optimizer state dict (keyed by parameter name or by integer id with ``param_names``) into the live,
    sharded optimizer: every rank keeps the ranges of its shards (the reference's function of this name,
    ``olmo/checkpoint.py:202-216``)."""
    FullCheckpointer.load_optim_state_into(dist_model, optim, FullCheckpointer._normalise_optim_state(optim_state, {}))


class TorchNewStyleShardedCheckpointer(Checkpointer):
    """Reads *and writes* the reference's ``torch_new`` sharded layout (``olmo/checkpoint.py:892-966``): ``model_and_optim/``
    through the two functions above plus ``train/rank{r}.pt`` per rank.  Selected by ``sharded_checkpointer: torch_new``
    together with ``OLMO_B200_WRITE_REFERENCE_LAYOUT=1`` (otherwise that value, like the others, writes the flat-shard
    format, which saves without gathering anything to one rank)."""

    def save_checkpoint(self, dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, trainer_state: Dict[str, Any], *, upload_to: Optional[str] = None) -> None:
        with self._temporary_wd(dir) as tmp:
            save_fsdp_model_and_optim_state(tmp, dist_model, optim, upload_to=upload_to, save_overwrite=self.cfg.save_overwrite)
            save_state_dict(tmp, f"train/rank{get_global_rank()}.pt", trainer_state, upload_to=upload_to, save_overwrite=self.cfg.save_overwrite,
                            synchronize=False)
            self._save_config(tmp, upload_to=upload_to)

    def restore_checkpoint(
        self, load_path: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, local_cache: Optional[PathOrStr] = None,
        load_optimizer_state: bool = True,
    ) -> Dict[str, Any]:
        load_fsdp_model_and_optim_state(load_path, dist_model, optim, local_cache=local_cache, load_optimizer_state=load_optimizer_state)
        try:
            return load_state_dict(load_path, f"train/rank{get_global_rank()}.pt", local_cache=local_cache)
        except FileNotFoundError:
            return load_state_dict(load_path, "train/rank0.pt", local_cache=local_cache)  # written by a smaller job

    def unshard_checkpoint(
        self, load_path: PathOrStr, *, local_cache: Optional[PathOrStr] = None, load_optimizer_state: bool = True,
        load_trainer_state: bool = True, device: Optional[torch.device] = None,
    ) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
        return unshard_torch_dcp_checkpoint(load_path, load_optimizer_state=load_optimizer_state, load_trainer_state=load_trainer_state)


class _ReferenceLayoutReader(Checkpointer):
    """Read-only checkpointer for one sharded layout of the reference implementation (:mod:`olmo_b200.checkpoint_compat`
    does the work).  These layouts serialise FSDP1 objects this engine does not have, so ``save_checkpoint`` refuses and
    names the two ways of producing a checkpoint the reference loads."""

    layout = ""

    def save_checkpoint(self, dir: PathOrStr, dist_model: nn.Module, optim: Optimizer, trainer_state: Dict[str, Any], *, upload_to: Optional[str] = None) -> None:
        raise OLMoCheckpointError(
            f"the '{self.layout}' layout is read-only here; save an unsharded checkpoint (both implementations read it) or write the "
            "'torch_new' layout (TorchNewStyleShardedCheckpointer, scripts/export_sharded.py)"
        )

    def restore_checkpoint(
        self, load_path: PathOrStr, dist_model: nn.Module, optim: Optimizer, *, local_cache: Optional[PathOrStr] = None,
        load_optimizer_state: bool = True,
    ) -> Dict[str, Any]:
        return FlatShardCheckpointer(self.cfg)._restore_foreign(load_path, self.layout, dist_model, optim, load_optimizer_state=load_optimizer_state)

    def unshard_checkpoint(
        self, load_path: PathOrStr, *, local_cache: Optional[PathOrStr] = None, load_optimizer_state: bool = True,
        load_trainer_state: bool = True, device: Optional[torch.device] = None,
    ) -> Tuple[Dict[str, torch.Tensor], Optional[Dict[str, Any]], Optional[Dict[str, Any]]]:
        from .checkpoint_compat import unshard_reference_checkpoint

        return unshard_reference_checkpoint(load_path, layout=self.layout, load_optimizer_state=load_optimizer_state,
                                            load_trainer_state=load_trainer_state, device=device)


class TorchLegacyShardedCheckpointer(_ReferenceLayoutReader):
    """``rank{r}.pt`` files of pickled ``ShardedTensor`` objects (the reference's default, ``olmo/checkpoint.py:969-1453``)."""

    layout = "torch_legacy"


class LocalShardedCheckpointer(_ReferenceLayoutReader):
    """Raw FSDP flat-parameter pieces per rank (``olmo/checkpoint.py:1474-1906``)."""

    layout = "local"


class OlmoCoreCheckpointer(_ReferenceLayoutReader):
    """The layout written through the ``olmo_core`` package (``olmo/checkpoint.py:1909-2014``): reading it needs that
    package's own loader, which is not bundled; every operation says so."""

    layout = "olmo_core"


def build_sharded_checkpointer(cfg: TrainConfig, *, name: Optional[ShardedCheckpointerType] = None, use_shared_mem_impl: bool = False) -> Checkpointer:
    """The sharded checkpointer of this framework.

    ``sharded_checkpointer`` (``torch_new``, ``torch_legacy``, ``local``, ``olmo_core``) names layouts of the reference's
    FSDP1 checkpointers.  This engine has no FSDP1 flat parameters or ``ShardedTensor`` objects to serialise, so by
    default every value *writes* the one flat-shard layout described in :class:`FlatShardCheckpointer`; the key is
    accepted so that reference configs load unchanged.  The exception is opt-in: ``torch_new`` together with
    ``OLMO_B200_WRITE_REFERENCE_LAYOUT=1`` in the environment selects :class:`TorchNewStyleShardedCheckpointer`, which
    writes the reference's ``torch_new`` layout.  On the *read* side the layout of a directory is detected, and checkpoints written
    by the reference in the ``torch_new``, ``torch_legacy`` and ``local`` layouts are restored, resharded or unsharded
    (:mod:`olmo_b200.checkpoint_compat`); ``olmo_core`` directories raise an error that says what to do."""
    del use_shared_mem_impl
    chosen = name if name is not None else cfg.sharded_checkpointer
    wants_reference = os.environ.get("OLMO_B200_WRITE_REFERENCE_LAYOUT", "0").strip().lower() in ("1", "true", "yes", "on")
    if wants_reference and str(getattr(chosen, "value", chosen)) == "torch_new":
        return TorchNewStyleShardedCheckpointer(cfg)
    return FlatShardCheckpointer(cfg)
