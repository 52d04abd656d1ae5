"""
Training loop (reference: ``olmo/train.py:67-1396``).

The public surface is the reference's — :class:`Trainer` with ``fit``, ``train_step``, ``eval``,
``save_checkpoint``, ``restore_checkpoint`` and the trainer-state dict layout — while the step itself has two
implementations chosen per model:

* the *fused* step drives :meth:`FlatShardEngine.train_microbatch` (explicit forward/backward kernel
  sequences, fp32 gradients written by GEMM epilogues, whole-shard optimizer kernels), timed on the device with
  CUDA events;
* the *portable* step is ordinary autograd under autocast, for CPU runs and for configurations outside the
  kernels' coverage.
"""
from __future__ import annotations

import cProfile
import functools
import gc
import logging
import math
import os
import random
import shutil
import time
from collections import deque
from dataclasses import dataclass, field
from itertools import islice
from pathlib import Path
from pstats import SortKey
from typing import Any, Callable, Deque, Dict, List, Optional, TextIO, Tuple, Union

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch.utils.data import DataLoader

from .aliases import PathOrStr
from .checkpoint import Checkpointer, FullCheckpointer, build_sharded_checkpointer
from .config import (
    CheckpointType,
    DDPGradSyncMode,
    DistributedStrategy,
    SchedulerUnits,
    ShardedCheckpointerType,
    SpeedMonitorConfig,
    TrainConfig,
)
from .data import IterableDataset
from .eval import Evaluator
from .exceptions import OLMoConfigurationError
from .models.olmo import OLMo
from .ops.loss import cross_entropy_loss, fused_cross_entropy
from .optim import Optimizer, Scheduler
from .torch_util import (
    barrier,
    gc_cuda,
    get_fs_local_rank,
    get_global_rank,
    get_world_size,
    is_distributed,
    move_to_device,
    nvtx_range,
    peak_gpu_memory,
    synchronize_flag,
    synchronize_value,
)
from .util import upload

__all__ = ["SpeedMonitor", "LRMonitor", "Trainer", "cross_entropy_loss", "fused_loss_fn"]

log = logging.getLogger(__name__)

fused_loss_fn = fused_cross_entropy


def _wandb_run():
    try:
        import wandb

        return wandb.run
    except Exception:
        return None


def _wandb_log(metrics: Dict[str, Any], step: int) -> None:
    if _wandb_run() is not None:
        import wandb

        wandb.log(metrics, step=step)


@dataclass
class SpeedMonitor:
    """Windowed throughput.  Besides the reference's host-clock figures it reports model FLOP utilisation when
    ``gpu_flops_available`` is configured."""

    cfg: SpeedMonitorConfig
    start_times: Deque[float] = field(default_factory=lambda: deque([]))
    global_total_tokens: int = 0
    total_training_Gflops: float = 0
    device_interval_tokens: Deque[int] = field(default_factory=lambda: deque([]))
    _flops_per_token: float = 0.0

    def batch_start(
        self, global_total_tokens: int, device_batch_num_tokens: int, num_fwd_flops: int, num_bck_flops: int, record: bool = True
    ) -> None:
        self.global_total_tokens = global_total_tokens
        self._flops_per_token = float(num_fwd_flops + num_bck_flops)
        self.total_training_Gflops += (num_fwd_flops + num_bck_flops) * device_batch_num_tokens * get_world_size() / 1e9
        if record:
            if len(self.start_times) >= self.cfg.window_size:
                self.start_times.popleft()
                self.device_interval_tokens.popleft()
            self.start_times.append(time.monotonic())
            self.device_interval_tokens.append(device_batch_num_tokens)

    def reset(self) -> None:
        self.start_times.clear()
        self.device_interval_tokens.clear()

    def check(self) -> Dict[str, float]:
        metrics: Dict[str, float] = {"throughput/total_tokens": self.global_total_tokens}
        if self.total_training_Gflops > 0:
            metrics["throughput/total_training_Gflops"] = self.total_training_Gflops
            metrics["throughput/total_training_log_Gflops"] = math.log(self.total_training_Gflops)
        if self.start_times:
            elapsed = time.monotonic() - self.start_times[0]
            tps = sum(self.device_interval_tokens) / elapsed
            metrics["throughput/device/tokens_per_second"] = tps
            metrics["throughput/device/batches_per_second"] = len(self.start_times) / elapsed
            if self.cfg.gpu_flops_available:
                metrics["throughput/device/mfu"] = tps * self._flops_per_token / float(self.cfg.gpu_flops_available)
        return metrics


@dataclass
class LRMonitor:
    optim: torch.optim.Optimizer

    def check(self) -> Dict[str, float]:
        return {f"optim/learning_rate_group{i}": g["lr"] for i, g in enumerate(self.optim.param_groups)}


def _fmt(value: float) -> str:
    if value < 0.0001:
        return str(value)
    if value > 1000:
        return f"{int(value):,d}"
    if value > 100:
        return f"{value:.1f}"
    if value > 10:
        return f"{value:.2f}"
    if value > 1:
        return f"{value:.3f}"
    return f"{value:.4f}"


@dataclass
class Trainer:
    cfg: TrainConfig
    model: OLMo
    dist_model: torch.nn.Module  # ShardedModel or SingleAccelerator
    optim: Optimizer
    scheduler: Scheduler
    train_loader: DataLoader
    device: torch.device
    evaluators: List[Evaluator]
    epoch: Optional[int] = None
    global_step: int = 0
    global_train_examples_seen_this_epoch: int = 0  # restarts at 0 each epoch; this is the data-loader position
    global_train_tokens_seen: int = 0
    checkpoints: List[Path] = field(default_factory=list)
    unsharded_checkpoints: List[Path] = field(default_factory=list)
    ephemeral_checkpoints: List[Path] = field(default_factory=list)
    min_train_loss: float = float("inf")
    cur_train_loss: float = float("inf")
    indices_file: Optional[TextIO] = None
    _start_time: float = 0.0
    _gc_init_state: bool = True
    loss_fn: Callable[..., torch.Tensor] = field(default_factory=lambda: cross_entropy_loss)  # type: ignore
    last_sharded_checkpoint_step: Optional[int] = None
    last_unsharded_checkpoint_step: Optional[int] = None
    last_step_device_ms: Optional[float] = None  # device time of the most recent train_step (CUDA events)

    def __post_init__(self) -> None:
        if self.cfg.fused_loss and self.device.type == "cuda":
            self.loss_fn = fused_cross_entropy  # type: ignore[assignment]
        self._engine = getattr(self.dist_model, "engine", None)
        self._fused = bool(self._engine is not None and self._engine.fused)
        self._pinned: Dict[str, torch.Tensor] = {}

    # ------------------------------------------------------------------------------ accounting
    @property
    def dataset(self) -> IterableDataset:
        assert isinstance(self.train_loader.dataset, IterableDataset)
        return self.train_loader.dataset

    @property
    def tokens_per_batch(self) -> int:
        return self.cfg.global_train_batch_size * self.cfg.model.max_sequence_length

    @property
    def batches_per_epoch(self) -> int:
        return self.dataset.total_size // self.cfg.global_train_batch_size

    @property
    def max_epochs(self) -> int:
        d = self.cfg.max_duration
        return int(d[:-2].strip()) if isinstance(d, str) and d.endswith("ep") else 1

    def _duration(self) -> Tuple[str, int]:
        d = self.cfg.max_duration
        if isinstance(d, int):
            return "steps", d
        if isinstance(d, str):
            if d.endswith("T"):
                return "tokens", int(float(d[:-1].strip()))
            if d.endswith("ep"):
                return "epochs", int(d[:-2].strip())
            return "steps", int(float(d))
        raise TypeError(f"expected int or str for 'max_duration', found {type(d)}")

    @property
    def max_steps(self) -> int:
        unit, n = self._duration()
        if unit == "steps":
            return n
        if unit == "tokens":
            remaining = max(n - self.global_train_tokens_seen, 0)
            return self.global_step + math.ceil(remaining / self.tokens_per_batch)
        return n * self.batches_per_epoch

    @property
    def max_tokens(self) -> int:
        unit, n = self._duration()
        if unit == "tokens":
            return n
        if unit == "epochs":
            return n * self.batches_per_epoch * self.tokens_per_batch
        return self.global_train_tokens_seen + max(n - self.global_step, 0) * self.tokens_per_batch

    @property
    def scheduler_current(self) -> int:
        return self.global_step if self.cfg.scheduler.units == SchedulerUnits.steps else self.global_train_tokens_seen

    @property
    def scheduler_max(self) -> int:
        return self.max_steps if self.cfg.scheduler.units == SchedulerUnits.steps else self.max_tokens

    # ----------------------------------------------------------------------------- trainer state
    def trainer_state_dict(self) -> Dict[str, Any]:
        """Plain containers only, so the reference can unpickle it (``olmo/train.py:322-339``)."""
        return {
            "epoch": self.epoch or 0,
            "global_step": self.global_step,
            "global_train_examples_seen_this_epoch": self.global_train_examples_seen_this_epoch,
            "global_train_tokens_seen": self.global_train_tokens_seen,
            "world_size": get_world_size(),
            "checkpoints": self.checkpoints,
            "unsharded_checkpoints": self.unsharded_checkpoints,
            "ephemeral_checkpoints": self.ephemeral_checkpoints,
            "rng": {
                "python": random.getstate(),
                "numpy": np.random.get_state(),
                "torch": torch.random.get_rng_state(),
                "cuda": torch.cuda.get_rng_state() if torch.cuda.is_available() else None,
                "mps": None,
            },
        }

    def _own_checkpoints(self, paths: List[Any]) -> List[Path]:
        root = Path(self.cfg.save_folder).resolve()
        return [Path(p) for p in paths if Path(p).is_dir() and Path(p).resolve().parent == root]

    def load_trainer_state_dict(self, state_dict: Dict[str, Any]) -> None:
        self.checkpoints = self._own_checkpoints(state_dict["checkpoints"])
        self.unsharded_checkpoints = self._own_checkpoints(state_dict["unsharded_checkpoints"])
        self.ephemeral_checkpoints = self._own_checkpoints(state_dict.get("ephemeral_checkpoints", []))

        saved_epoch = state_dict.get("epoch") or 0
        self.global_step = state_dict["global_step"]
        legacy_steps = state_dict.get("global_data_step", self.global_step)
        self.global_train_examples_seen_this_epoch = state_dict.get(
            "global_train_examples_seen_this_epoch",
            state_dict.get("global_train_examples_seen", legacy_steps * self.cfg.global_train_batch_size),
        )
        self.global_train_tokens_seen = state_dict.get(
            "global_train_tokens_seen", legacy_steps * self.cfg.global_train_batch_size * self.cfg.model.max_sequence_length
        )
        if not self.cfg.restore_dataloader:
            self.epoch = 0
            self.global_step = 0
            self.global_train_tokens_seen = 0
            self.global_train_examples_seen_this_epoch = 0
        elif self.epoch is None:
            self.epoch = saved_epoch
        elif saved_epoch != self.epoch:
            log.info("Starting new epoch (epoch = %s)", self.epoch)
            self.global_train_examples_seen_this_epoch = 0
        assert self.epoch is not None
        if self.dataset.epoch != self.epoch:
            log.info("Reshuffling data loader for epoch %d...", self.epoch)
            self.dataset.reshuffle(self.epoch)
        if self.cfg.fast_forward_batches:
            log.info("Fast-forwarding data loader by %d steps", self.cfg.fast_forward_batches)
            self.global_train_examples_seen_this_epoch += self.cfg.fast_forward_batches * self.cfg.global_train_batch_size
        if self.global_train_examples_seen_this_epoch > 0:
            log.info("Data loader will start at instance index %d", self.global_train_examples_seen_this_epoch)
            self.dataset.start_index = self.global_train_examples_seen_this_epoch

        # LR and weight decay always come from the *current* config, not from the checkpoint
        lr = self.scheduler.get_lr(self.cfg.optimizer.learning_rate, self.scheduler_current, self.scheduler_max)
        for group in self.optim.param_groups:
            group["lr"] = lr
            group["initial_lr"] = self.cfg.optimizer.learning_rate
            if group.get("weight_decay", 0.0) > 0.0:
                group["weight_decay"] = self.cfg.optimizer.weight_decay

        if "rng" in state_dict and state_dict.get("world_size", get_world_size()) == get_world_size():
            log.info("Restoring RNG states...")
            self.restore_rng_state(state_dict["rng"])
        else:
            log.warning(
                "Trainer will not restore RNG states since the RNG states in the checkpoint are missing or invalid. "
                "This typically happens when restoring from an unsharded checkpoint or a checkpoint that was saved "
                "with a different world size. If that's the case you can safely ignore this warning."
            )

    def restore_rng_state(self, rng_state: Dict[str, Any]) -> None:
        random.setstate(rng_state["python"])
        np.random.set_state(rng_state["numpy"])
        torch.set_rng_state(rng_state["torch"])
        if torch.cuda.is_available():
            if rng_state.get("cuda") is not None:
                torch.cuda.set_rng_state(rng_state["cuda"])
            else:
                log.warning("CUDA is available, but no RNG state was provided.")

    # ------------------------------------------------------------------------------ checkpoints
    def _checkpoint_kind(self, kind: CheckpointType) -> Tuple[str, List[Path], bool, int]:
        if kind == CheckpointType.sharded:
            return "", self.checkpoints, get_fs_local_rank() == 0, self.cfg.save_num_checkpoints_to_keep
        if kind == CheckpointType.unsharded:
            return "-unsharded", self.unsharded_checkpoints, get_global_rank() == 0, self.cfg.save_num_unsharded_checkpoints_to_keep
        if kind == CheckpointType.sharded_ephemeral:
            return "", self.ephemeral_checkpoints, get_fs_local_rank() == 0, 1
        raise NotImplementedError(kind)

    def _save_checkpoint(self, checkpointer: Checkpointer, kind: CheckpointType) -> Tuple[PathOrStr, Optional[PathOrStr]]:
        suffix, current, link_latest, keep = self._checkpoint_kind(kind)
        self._zero_grad()
        if self.indices_file is not None:
            self.indices_file.flush()
        ckpt_dir = Path(self.cfg.save_folder) / f"step{self.global_step}{suffix}"
        remote: Optional[str] = None
        if self.cfg.remote_save_folder is not None:
            remote = f"{self.cfg.remote_save_folder.rstrip('/')}/{ckpt_dir.name}"
        current.append(ckpt_dir)  # before the save: the trainer state that is written lists this checkpoint too
        try:
            checkpointer.save_checkpoint(ckpt_dir, self.dist_model, self.optim, self.trainer_state_dict(), upload_to=remote)
        except BaseException as e:
            # a save that did not complete (full disk, remote store down, rank lost) must not stay on the books: the
            # rotation below would count it, and a retry of the same step would list it twice
            current.remove(ckpt_dir)
            if isinstance(e, FileExistsError):
                raise OLMoConfigurationError(f"Checkpoint for step {self.global_step} already exists, use --save_overwrite to overwrite it")
            raise
        if link_latest:
            latest = Path(self.cfg.save_folder) / f"latest{suffix}"
            latest.unlink(missing_ok=True)
            try:
                latest.symlink_to(ckpt_dir.name, target_is_directory=True)
            except FileExistsError:
                if latest.resolve().name != ckpt_dir.name:  # another rank on a shared filesystem may have won
                    raise
        if keep > 0:
            while len(current) > keep:
                self.remove_checkpoint(0, kind)
        barrier()
        return (remote, ckpt_dir) if remote is not None else (ckpt_dir, None)

    def save_sharded_checkpoint(self):
        result = self._save_checkpoint(build_sharded_checkpointer(self.cfg), CheckpointType.sharded)
        self.last_sharded_checkpoint_step = self.global_step
        return result

    def save_ephemeral_checkpoint(self):
        result = self._save_checkpoint(build_sharded_checkpointer(self.cfg), CheckpointType.sharded_ephemeral)
        self.last_sharded_checkpoint_step = self.global_step
        return result

    def save_unsharded_checkpoint(self):
        result = self._save_checkpoint(FullCheckpointer(self.cfg), CheckpointType.unsharded)
        self.last_unsharded_checkpoint_step = self.global_step
        return result

    def save_checkpoint(self, checkpoint_type: CheckpointType = CheckpointType.sharded) -> Tuple[PathOrStr, Optional[PathOrStr]]:
        if checkpoint_type == CheckpointType.sharded:
            result = self.save_sharded_checkpoint()
        elif checkpoint_type == CheckpointType.unsharded:
            result = self.save_unsharded_checkpoint()
        elif checkpoint_type == CheckpointType.sharded_ephemeral:
            result = self.save_ephemeral_checkpoint()
        else:
            raise NotImplementedError(checkpoint_type)
        gc_cuda()
        return result

    def _remove(self, idx: int, checkpoints: List[Path], latest_name: str, writer: bool) -> None:
        oldest = checkpoints.pop(idx)
        barrier()
        if writer and oldest.is_dir():
            shutil.rmtree(oldest, ignore_errors=True)
            latest = Path(self.cfg.save_folder) / latest_name
            if latest.is_symlink() and latest.resolve() == oldest.resolve():
                latest.unlink()
        barrier()

    def remove_sharded_checkpoint(self, idx: int = 0) -> None:
        self._remove(idx, self.checkpoints, "latest", get_fs_local_rank() == 0)

    def remove_ephemeral_checkpoint(self, idx: int = 0) -> None:
        self._remove(idx, self.ephemeral_checkpoints, "latest", get_fs_local_rank() == 0)

    def remove_unsharded_checkpoint(self, idx: int = 0) -> None:
        self._remove(idx, self.unsharded_checkpoints, "latest-unsharded", get_global_rank() == 0)

    def remove_checkpoint(self, idx: int = 0, checkpoint_type: CheckpointType = CheckpointType.sharded) -> None:
        {
            CheckpointType.sharded: self.remove_sharded_checkpoint,
            CheckpointType.unsharded: self.remove_unsharded_checkpoint,
            CheckpointType.sharded_ephemeral: self.remove_ephemeral_checkpoint,
        }[checkpoint_type](idx)

    def _restore(self, checkpointer: Checkpointer, load_path, local_cache, load_optimizer_state, load_trainer_state) -> None:
        self._zero_grad()
        state = checkpointer.restore_checkpoint(
            load_path, self.dist_model, self.optim, local_cache=local_cache, load_optimizer_state=load_optimizer_state
        )
        if load_trainer_state:
            self.load_trainer_state_dict(state)
        barrier()

    def restore_sharded_checkpoint(
        self, load_path: PathOrStr, local_cache: Optional[PathOrStr] = None, *, load_optimizer_state: bool = True,
        load_trainer_state: bool = True, sharded_checkpointer: Optional[ShardedCheckpointerType] = None,
    ) -> None:
        self._restore(build_sharded_checkpointer(self.cfg, name=sharded_checkpointer), load_path, local_cache, load_optimizer_state, load_trainer_state)

    def restore_unsharded_checkpoint(
        self, load_path: PathOrStr, local_cache: Optional[PathOrStr] = None, *, load_optimizer_state: bool = True,
        load_trainer_state: bool = True,
    ) -> None:
        self._restore(FullCheckpointer(self.cfg), load_path, local_cache, load_optimizer_state, load_trainer_state)

    def restore_checkpoint(
        self, load_path: PathOrStr, *, checkpoint_type: Optional[CheckpointType] = None, local_cache: Optional[PathOrStr] = None,
        load_optimizer_state: bool = True, load_trainer_state: bool = True,
        sharded_checkpointer: Optional[ShardedCheckpointerType] = None,
    ) -> None:
        unsharded = checkpoint_type == CheckpointType.unsharded or (
            checkpoint_type is None and str(load_path).rstrip("/").endswith("-unsharded")
        )
        if unsharded:
            self.restore_unsharded_checkpoint(load_path, local_cache, load_optimizer_state=load_optimizer_state, load_trainer_state=load_trainer_state)
        elif checkpoint_type in (None, CheckpointType.sharded):
            self.restore_sharded_checkpoint(
                load_path, local_cache, load_optimizer_state=load_optimizer_state, load_trainer_state=load_trainer_state,
                sharded_checkpointer=sharded_checkpointer,
            )
        else:
            raise NotImplementedError(checkpoint_type)
        gc_cuda()

    # -------------------------------------------------------------------------- module tracing
    def _setup_module_output_save_hooks(self, micro_batch_idx: int) -> List[Any]:
        """On the configured steps dump every module's first input and output of micro-batch 0 (rank 0) to
        ``traces/step{N}/``; such steps run on the portable path so that every module is a real call."""
        steps = self.cfg.module_outputs_save_steps
        if steps is None or self.global_step not in steps or micro_batch_idx != 0 or get_global_rank() != 0:
            return []
        folder = Path(self.cfg.save_folder) / f"traces/step{self.global_step}"
        if folder.exists():
            if not self.cfg.save_overwrite:
                raise OLMoConfigurationError(f"Attempting to overwrite traces at step {self.global_step} without --save_overwrite")
            shutil.rmtree(folder)
        folder.mkdir(parents=True)

        def hook(name: str, _module, args, output) -> None:
            first = args[0] if len(args) > 0 else torch.tensor(())
            n = 0
            while (inp := folder / f"{name}_{n}_input.pt").exists():
                n += 1
            torch.save(first, inp)
            torch.save(output, folder / f"{name}_{n}_output.pt")

        return [m.register_forward_hook(functools.partial(hook, name)) for name, m in self.model.named_modules(prefix="model")]

    # ------------------------------------------------------------------------------------ step
    def get_labels(self, batch: Dict[str, Any]) -> torch.Tensor:
        """Next-token targets ``(B, T-1)`` with ``-100`` where the label mask, attention mask or instance mask
        excludes a position."""
        labels = batch["input_ids"].clone()
        if (label_mask := batch.get("label_mask")) is not None:
            labels.masked_fill_(~label_mask, -100)
        if (attention_mask := batch.get("attention_mask")) is not None:
            labels.masked_fill_(attention_mask == 0.0, -100)
        if (instance_mask := batch.get("instance_mask")) is not None:
            labels.masked_fill_(~instance_mask.unsqueeze(-1), value=-100)
        return labels[..., 1:].contiguous()

    def model_forward(
        self, batch: Dict[str, Any], loss_reduction: str = "mean", compute_z_loss: bool = False
    ) -> Tuple[torch.Tensor, Optional[torch.Tensor], torch.Tensor]:
        logits = self.dist_model(
            input_ids=batch["input_ids"],
            attention_mask=batch.get("attention_mask"),
            attention_bias=batch.get("attention_bias"),
            doc_lens=batch.get("doc_lens"),
            max_doc_lens=batch.get("max_doc_lens"),
        ).logits
        flat = logits[..., :-1, :].contiguous().view(-1, logits.size(-1))
        labels = self.get_labels(batch).view(-1)
        ce_loss, z_loss = self.loss_fn(flat, labels, ignore_index=-100, reduction=loss_reduction, compute_z_loss=compute_z_loss)
        if loss_reduction == "none":
            ce_loss = ce_loss.view(batch["input_ids"].shape[0], -1)
            if z_loss is not None:
                z_loss = z_loss.view(batch["input_ids"].shape[0], -1)
        return ce_loss, z_loss, logits

    def train_micro_batch(self, micro_batch: Dict[str, Any], batch_size_in_tokens: int):
        # NOTE: like the reference, the z-loss multiplier used here is the loss function's default (1e-4);
        # `auxiliary_loss_multiplier` from the config is not consulted (olmo/train.py:749-751).
        ce_loss, z_loss, logits = self.model_forward(micro_batch, compute_z_loss=self.cfg.softmax_auxiliary_loss, loss_reduction="sum")
        ce_loss = ce_loss / batch_size_in_tokens
        if self.cfg.softmax_auxiliary_loss:
            assert z_loss is not None
            z_loss = z_loss / batch_size_in_tokens
            loss = ce_loss + z_loss
        else:
            loss = ce_loss
        del logits
        return loss, ce_loss, z_loss

    def _fused_step_usable(self, batch: Dict[str, Any]) -> bool:
        if not self._fused:
            return False
        if batch.get("attention_mask") is not None and not bool(torch.all(batch["attention_mask"] == 1)):
            return False
        if batch.get("attention_bias") is not None:
            return False
        if batch.get("doc_lens") is not None:  # document masking needs the native attention kernel's shape coverage
            mc = self.cfg.model
            if mc.d_model // mc.n_heads > 128:
                return False
        steps = self.cfg.module_outputs_save_steps
        return not (steps is not None and self.global_step in steps)

    @staticmethod
    def _doc_start(batch: Dict[str, Any]) -> Optional[torch.Tensor]:
        """Per-token document starts for intra-document masking on the fused path (``None`` without ``doc_lens``)."""
        doc_lens = batch.get("doc_lens")
        if doc_lens is None:
            return None
        from .ops.attention_native import doc_start_from_lengths

        return doc_start_from_lengths(doc_lens, batch["input_ids"].shape[1])

    def _labels_aligned(self, batch: Dict[str, Any]) -> torch.Tensor:
        """``(B, T)`` labels where entry ``t`` is the target of position ``t`` (last position ignored)."""
        shifted = self.get_labels(batch)
        return F.pad(shifted, (0, 1), value=-100)

    def train_batch(self, batch: Dict[str, Any]) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        micro_batches = self.split_batch(batch)
        batch_size_in_tokens = batch["input_ids"].numel()
        fused = self._fused_step_usable(batch)
        if self._fused and not fused:
            # a fused engine keeps no autograd graph (its module parameters do not require gradients)
            raise OLMoConfigurationError(
                "this batch cannot run on the fused kernel path (attention mask with padding, attention bias, document "
                "lengths with a head dimension above 128, or a module-output trace step) and "
                "the engine was built for it; build the engine with force_portable=True (set OLMO_B200_KERNELS=0) for such data"
            )
        del batch
        ce_batch_loss = torch.tensor(0.0, device=self.device)
        z_batch_loss = torch.tensor(0.0, device=self.device) if self.cfg.softmax_auxiliary_loss else None
        n = len(micro_batches)
        for idx, mb in enumerate(micro_batches):
            if fused:
                ce, z = self._engine.train_microbatch(
                    mb["input_ids"], self._labels_aligned(mb), float(batch_size_in_tokens),
                    z_mult=1e-4 if self.cfg.softmax_auxiliary_loss else 0.0,
                    ac_strategy=self.model.activation_checkpointing_strategy,
                    is_last=idx == n - 1,
                    doc_start=self._doc_start(mb),
                )
                ce_batch_loss += ce
                if z_batch_loss is not None:
                    z_batch_loss += z
                continue
            hooks = self._setup_module_output_save_hooks(idx)
            autocast_on = self.cfg.precision not in (None, "fp32")
            ac_device = self.device.type if self.device.type in ("cuda", "cpu", "mps") else "cuda"
            with torch.autocast(ac_device, enabled=autocast_on, dtype=self.cfg.autocast_precision if autocast_on else None):
                loss, ce_loss, z_loss = self.train_micro_batch(mb, batch_size_in_tokens)
                ce_batch_loss += ce_loss.detach()
                if z_loss is not None and z_batch_loss is not None:
                    z_batch_loss += z_loss.detach()
            loss.backward()
            if self._engine is not None:
                self._engine.note_microbatch_backward()
                if (
                    self.cfg.distributed_strategy == DistributedStrategy.ddp and self.cfg.ddp is not None
                    and self.cfg.ddp.grad_sync_mode == DDPGradSyncMode.micro_batch
                ):
                    self._engine.finish_grad_sync()
            for h in hooks:
                h.remove()
        return ce_batch_loss, z_batch_loss

    def _zero_grad(self) -> None:
        if self._engine is not None:
            self._engine.zero_grad()
        else:
            self.optim.zero_grad(set_to_none=True)

    def _stage_batch(self, batch: Dict[str, Any]) -> Dict[str, Any]:
        """Host -> device copy of a batch.  On CUDA the source is staged through pinned buffers that persist
        across steps so the copy is asynchronous with respect to the host."""
        if self.device.type != "cuda":
            return move_to_device(batch, self.device)
        out: Dict[str, Any] = {}
        for key, value in batch.items():
            if isinstance(value, torch.Tensor) and not value.is_cuda:
                if not value.is_pinned():
                    buf = self._pinned.get(key)
                    if buf is None or buf.shape != value.shape or buf.dtype != value.dtype:
                        buf = torch.empty(value.shape, dtype=value.dtype, pin_memory=True)
                        self._pinned[key] = buf
                    buf.copy_(value)
                    value = buf
                out[key] = value.to(self.device, non_blocking=True)
            else:
                out[key] = move_to_device(value, self.device)
        return out

    def train_step(self, batch: Dict[str, Any], reduce_global_loss: bool = True) -> Dict[str, float]:
        metrics: Dict[str, float] = {}
        if self.indices_file is not None and "index" in batch:
            self.indices_file.write(f"{self.global_step}\t" + "\t".join(str(int(i)) for i in batch["index"]) + "\n")
        if (instance_mask := batch.get("instance_mask")) is not None:
            metrics["train/masked_instances_local_rank"] = (~instance_mask).sum().item()

        timed = self.device.type == "cuda"
        if timed:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        self._zero_grad()
        with nvtx_range("stage_batch"):
            batch = self._stage_batch(batch)
        with nvtx_range("forward_backward"):
            ce_batch_loss, z_batch_loss = self.train_batch(batch)

        if reduce_global_loss and is_distributed():
            dist.reduce(ce_batch_loss, 0)
            ce_batch_loss.div_(get_world_size())
            if z_batch_loss is not None:
                dist.reduce(z_batch_loss, 0)
                z_batch_loss.div_(get_world_size())

        collect = self.should_log_optim_metrics_this_step()
        with nvtx_range("clip_grads"):
            optim_metrics = self.optim.clip_grads_and_collect_metrics(
                self.global_step, collect_param_metrics=collect, process_group=getattr(self.dist_model, "process_group", None),
                device=self.device,
            )
        for group in self.optim.param_groups:
            group["lr"] = self.scheduler.get_lr(self.cfg.optimizer.learning_rate, self.scheduler_current, self.scheduler_max)
            group["max_grad_norm"] = self.scheduler.get_max_grad_norm(self.cfg.max_grad_norm, self.scheduler_current, self.scheduler_max)
            group["max_grad_norm_ratio"] = self.scheduler.get_max_grad_norm(self.cfg.max_grad_norm_ratio, self.scheduler_current, self.scheduler_max)
        with nvtx_range("optimizer_step"):
            self.optim.step()
        if timed:
            ev1.record()

        # one device -> host read brings back the losses (and, on the fused path, the kernel status word)
        self.cur_train_loss = ce_batch_loss.item()
        if math.isnan(self.cur_train_loss):
            raise ValueError("nan loss encountered")
        if z_batch_loss is not None:
            z = z_batch_loss.item()
            if math.isnan(z):
                raise ValueError("nan loss encountered")
            metrics["train/ZLoss"] = z
        if self._fused:
            from .ops import check_status

            check_status(self.device)
        if timed:
            self.last_step_device_ms = ev0.elapsed_time(ev1)
        for key, value in optim_metrics.items():
            metrics[f"optim/{key}"] = value.item()
        self.min_train_loss = min(self.min_train_loss, self.cur_train_loss)
        metrics["train/CrossEntropyLoss"] = self.cur_train_loss
        metrics["train/Perplexity"] = math.exp(self.cur_train_loss) if self.cur_train_loss < 700 else float("inf")
        if collect:
            for key, value in self.optim.get_post_step_metrics(self.dist_model, process_group=getattr(self.dist_model, "process_group", None)).items():
                metrics[f"optim/{key}"] = value.item()
        return metrics

    def eval_batch(self, batch: Dict[str, Any]) -> Tuple[torch.Tensor, torch.Tensor]:
        autocast_on = self.cfg.precision not in (None, "fp32")
        ac_device = self.device.type if self.device.type in ("cuda", "cpu", "mps") else "cuda"
        with torch.autocast(ac_device, enabled=autocast_on, dtype=self.cfg.autocast_precision if autocast_on else None):
            ce_loss, _, logits = self.model_forward(batch, loss_reduction="none")
        return ce_loss.mean(dim=-1), logits

    def eval_step(self, batch: Dict[str, Any], evaluator: Evaluator) -> None:
        batch = move_to_device(batch, self.device)
        with torch.no_grad(), nvtx_range("eval_step"):
            ce_loss, logits = self.eval_batch(batch)
        evaluator.update_metrics(batch, ce_loss, logits)
        barrier()

    def split_batch(self, batch: Dict[str, Any]) -> List[Dict[str, Any]]:
        mb = self.cfg.device_train_microbatch_size
        n = batch["input_ids"].shape[0]
        if n <= mb:
            return [batch]
        pieces = math.ceil(n / mb)
        out: List[Dict[str, Any]] = [dict() for _ in range(pieces)]
        for key, value in batch.items():
            if isinstance(value, torch.Tensor):
                for i, part in enumerate(value.split(mb, dim=0)):
                    out[i][key] = part
            elif isinstance(value, list):
                for i in range(pieces):
                    out[i][key] = value[mb * i : mb * (i + 1)]
            else:
                raise ValueError(f"unexpected item in batch: '{key}={value}'")
        return out

    def system_metrics(self) -> Dict[str, float]:
        metrics: Dict[str, float] = {}
        if self.global_step < 3 or self.global_step % 10 == 0:
            peak = peak_gpu_memory()
            if peak is not None:
                metrics["System/Peak GPU Memory (MB)"] = peak
        return metrics

    def log_metrics_to_console(self, prefix: str, metrics: Dict[str, float]) -> None:
        shown = [f"    {k}={_fmt(v)}" for k, v in metrics.items() if k == "optim/total_grad_norm" or not k.startswith("optim/")]
        log.info(prefix + "\n" + "\n".join(shown))

    def should_log_optim_metrics_this_step(self) -> bool:
        if self.cfg.wandb is None:
            return False
        interval = self.cfg.optimizer.metrics_log_interval
        interval = self.cfg.wandb.log_interval if interval is None else max(interval, self.cfg.wandb.log_interval)
        return self.global_step % interval == 0

    def should_log_this_step(self) -> bool:
        if self.global_step % self.cfg.console_log_interval == 0:
            return True
        return self.cfg.wandb is not None and self.global_step % self.cfg.wandb.log_interval == 0

    def eval(self) -> Dict[str, Any]:
        self._zero_grad()
        self.dist_model.eval()
        results: Dict[str, Any] = {}
        for evaluator in self.evaluators:
            log.info("Running evaluation for '%s'...", evaluator.label)
            evaluator.reset_metrics()
            batches = iter(evaluator.eval_loader)
            limit = evaluator.subset_num_batches if evaluator.subset_num_batches is not None else self.cfg.eval_subset_num_batches
            if limit > 0:
                limit = min(limit, len(evaluator.eval_loader))
                batches = islice(batches, limit)
            for i, batch in enumerate(batches):
                self.eval_step(batch, evaluator)
                if i + 1 == limit or (i + 1) % self.cfg.console_log_interval == 0:
                    log.info("[eval_step=%d/%s]", i + 1, limit)
            metrics = evaluator.compute_metrics()
            results.update(metrics)
            self.log_metrics_to_console(f"{evaluator.label}", metrics)
        return results

    def check_if_cancelled(self) -> Tuple[bool, int]:
        """Rank 0 decides (time limit, early-stopping factor, a ``cancel(l)ed`` tag on the W&B run); the decision
        and the number of extra steps are broadcast."""
        cancel, reason, extra = False, None, 0
        if get_global_rank() == 0:
            if self.cfg.time_limit is not None and time.time() - self._start_time >= self.cfg.time_limit:
                cancel, reason, extra = True, "time limit reached", self.cfg.extra_steps_after_cancel
            elif (
                self.cfg.early_stopping_factor is not None
                and self.global_step > self.cfg.scheduler.t_warmup
                and self.cur_train_loss > self.cfg.early_stopping_factor * self.min_train_loss
            ):
                cancel, reason = True, "early stopping from loss increase"
            elif _wandb_run() is not None and (api_key := os.environ.get("WANDB_API_KEY")) is not None:
                try:
                    import wandb

                    run = wandb.Api(api_key=api_key).run(wandb.run.path)
                    if any(tag.lower() in {"cancel", "canceled", "cancelled"} for tag in (run.tags or [])):
                        cancel, reason, extra = True, "Weights & Biases tag", self.cfg.extra_steps_after_cancel
                except Exception:
                    log.info("Failed to check if W&B run is cancelled, continuing run.")
        cancel = synchronize_flag(cancel, self.device)
        if cancel:
            extra = synchronize_value(extra, self.device)
            tail = f", stopping in {extra} more steps..." if extra > 0 else ""
            log.warning("Run canceled%s%s", f" due to {reason}" if reason else "", tail)
        return cancel, extra

    def fit(self) -> None:
        cfg = self.cfg
        if cfg.stop_after is not None:
            cfg.stop_at = self.global_step + cfg.stop_after if cfg.stop_at is None else min(cfg.stop_at, self.global_step + cfg.stop_after)
        if cfg.stop_at is None:
            cfg.stop_at = self.max_steps + 10
        self._start_time = time.time()
        self._gc_init_state = gc.isenabled()
        if cfg.gen1_gc_interval is not None:
            gc.disable()
        if cfg.load_path is not None and self.global_step > 0 and cfg.eval_on_load:
            _wandb_log(self.eval(), self.global_step)

        self.dist_model.train()
        assert cfg.device_train_batch_size is not None
        speed = SpeedMonitor(cfg.speed_monitor)
        lrs = LRMonitor(self.optim)
        sysm = self.system_metrics()
        if sysm:
            self.log_metrics_to_console("Pre-train system metrics", sysm)
            _wandb_log(sysm, 0)

        py_prof = cProfile.Profile() if cfg.python_profiling else None
        profiler = self._make_torch_profiler() if (cfg.torch_profiling and get_global_rank() == 0) else None
        first_batch, cancel_initiated, save_checkpoints = True, False, True
        stop_at: int = cfg.stop_at
        if profiler is not None:
            profiler.__enter__()
        try:
            for epoch in range(self.epoch or 0, self.max_epochs):
                exhausted = True
                for batch in self.train_loader:
                    batch_size, seq_len = batch["input_ids"].shape
                    assert seq_len == cfg.model.max_sequence_length
                    if batch_size != cfg.device_train_batch_size:
                        # the tail of an epoch that does not fill a device batch (the reference asserts here as well)
                        raise OLMoConfigurationError(
                            f"a training batch holds {batch_size} instances instead of {cfg.device_train_batch_size}: the epoch does not "
                            "divide into whole batches; set data.drop_last=true (as the published configs do) to skip the remainder"
                        )
                    global_batch = batch_size * get_world_size()
                    self.global_step += 1
                    self.global_train_examples_seen_this_epoch += global_batch
                    self.global_train_tokens_seen += global_batch * seq_len
                    speed.batch_start(
                        global_total_tokens=self.global_train_tokens_seen, device_batch_num_tokens=batch_size * seq_len,
                        num_fwd_flops=self.model.num_fwd_flops, num_bck_flops=self.model.num_bck_flops, record=not first_batch,
                    )
                    should_log = self.should_log_this_step()
                    metrics = self.train_step(batch, reduce_global_loss=should_log)
                    if should_log:
                        metrics.update(speed.check())
                        metrics.update(self.system_metrics())
                        metrics.update(lrs.check())
                        if self.last_step_device_ms is not None:
                            metrics["throughput/device/step_ms"] = self.last_step_device_ms
                    if self.global_step % cfg.console_log_interval == 0:
                        header = f"[step={self.global_step}/{self.max_steps},epoch={epoch}]"
                        if get_global_rank() == 0:
                            self.log_metrics_to_console(header, metrics)
                        else:
                            log.info(header)
                    if cfg.wandb is not None and self.global_step % cfg.wandb.log_interval == 0:
                        _wandb_log(metrics, self.global_step)

                    if not cancel_initiated and self.global_step % cfg.canceled_check_interval == 0:
                        cancel_initiated, extra = self.check_if_cancelled()
                        if cancel_initiated:
                            stop_at = min(stop_at, self.global_step + extra)

                    if cfg.distributed_strategy == DistributedStrategy.fsdp:
                        periodic = cfg.save_interval is not None and self.global_step % cfg.save_interval == 0 and cfg.save_num_checkpoints_to_keep != 0
                        if save_checkpoints and (cancel_initiated or periodic):
                            log.info("Saving checkpoint...")
                            path, _ = self.save_checkpoint(CheckpointType.sharded)
                            log.info("Checkpoint saved to %s", path)
                            while self.ephemeral_checkpoints:
                                self.remove_ephemeral_checkpoint()
                            speed.reset()
                            if cancel_initiated:
                                save_checkpoints = False
                        elif cfg.save_interval_ephemeral is not None and self.global_step % cfg.save_interval_ephemeral == 0:
                            log.info("Saving ephemeral checkpoint...")
                            path, _ = self.save_checkpoint(CheckpointType.sharded_ephemeral)
                            log.info("Checkpoint saved to %s", path)
                            speed.reset()
                    if (
                        save_checkpoints and cfg.save_interval_unsharded is not None
                        and self.global_step % cfg.save_interval_unsharded == 0 and cfg.save_num_unsharded_checkpoints_to_keep != 0
                    ):
                        log.info("Saving unsharded checkpoint...")
                        path, _ = self.save_checkpoint(CheckpointType.unsharded)
                        log.info("Unsharded checkpoint saved to %s", path)
                        speed.reset()

                    if not cancel_initiated and (self.global_step % cfg.eval_interval == 0 or self.global_step >= stop_at):
                        _wandb_log(self.eval(), self.global_step)
                        speed.reset()
                        self.dist_model.train()

                    first_batch = False
                    if profiler is not None:
                        profiler.step()
                    if self.global_step >= stop_at:
                        exhausted = False
                        break
                    if cfg.gen1_gc_interval is not None and self.global_step % cfg.gen1_gc_interval == 0:
                        gc.collect(1)
                    if py_prof is not None:
                        if self.global_step == 5:
                            py_prof.enable()
                        elif self.global_step == 8:
                            py_prof.disable()
                            py_prof.print_stats(sort=SortKey.CUMULATIVE)
                            py_prof = None
                if not exhausted:
                    break
                log.info("Training epoch complete")
                self.epoch = epoch + 1
                self.global_train_examples_seen_this_epoch = 0
                self.dataset.start_index = 0
                if self.epoch < self.max_epochs:
                    log.info("Reshuffling data loader for epoch %d...", self.epoch)
                    self.dataset.reshuffle(self.epoch)
        finally:
            if profiler is not None:
                profiler.__exit__(None, None, None)

        if save_checkpoints:
            if cfg.save_interval_unsharded is not None and self.last_unsharded_checkpoint_step != self.global_step:
                log.info("Saving final unsharded model checkpoint...")
                path, _ = self.save_checkpoint(CheckpointType.unsharded)
                log.info("Unsharded checkpoint saved to %s", path)
            elif (
                cfg.save_num_checkpoints_to_keep != 0 and self.last_sharded_checkpoint_step != self.global_step
                and cfg.distributed_strategy == DistributedStrategy.fsdp
            ):
                log.info("Saving final checkpoint...")
                path, _ = self.save_checkpoint(CheckpointType.sharded)
                log.info("Checkpoint saved to %s", path)

    def _make_torch_profiler(self):
        """Rank-0 ``torch.profiler`` window (wait 1, warm-up 5, record 3 steps) that logs the top kernels and writes a
        chrome trace under ``save_folder/profiler/``."""
        from torch.profiler import ProfilerActivity, profile, schedule

        def on_trace_ready(p) -> None:
            out_dir = Path(self.cfg.save_folder) / "profiler"
            out_dir.mkdir(exist_ok=True)
            log.info("Profile by total GPU time at step %d:\n%s", p.step_num, p.key_averages().table(sort_by="self_cuda_time_total", row_limit=32))
            log.info("Profile by total CPU time at step %d:\n%s", p.step_num, p.key_averages().table(sort_by="self_cpu_time_total", row_limit=32))
            trace = out_dir / f"{p.step_num}.chrome_trace.json.gz"
            p.export_chrome_trace(str(trace))
            if self.cfg.remote_save_folder is not None:
                upload(trace, f"{self.cfg.remote_save_folder.rstrip('/')}/profiler/{trace.name}")

        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
        return profile(activities=acts, record_shapes=False, profile_memory=False, with_stack=True,
                       schedule=schedule(wait=1, warmup=5, active=3, repeat=1), on_trace_ready=on_trace_ready)

    def close(self, exit_code: int = 0) -> None:
        gc_cuda()
        if self.indices_file is not None:
            self.indices_file.flush()
            self.indices_file.close()
        gc.enable() if self._gc_init_state else gc.disable()
        if _wandb_run() is not None:
            import wandb

            wandb.finish(exit_code=exit_code, quiet=True)

    def __enter__(self) -> "Trainer":
        return self

    def __exit__(self, exc_type, exc_val, exc_tb) -> None:
        del exc_val, exc_tb
        self.close(0 if exc_type is None else 1)
