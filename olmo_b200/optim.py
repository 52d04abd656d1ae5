"""
Optimizers, gradient clipping with metric collection, and learning-rate schedules.

Capabilities follow the reference's ``olmo/optim.py:38-1040``; the implementation differs:

* per-parameter statistics are computed with batched ``torch._foreach_*`` calls and one stacked
  collective instead of one reduction per parameter;
* when the parameters are views into the flat fp32 shards of
  :class:`olmo_b200.parallel.fsdp.FlatShardEngine`, clipping and the AdamW / Lion update run as fused
  kernels over whole shards (``csrc/loss_optim.cu``): Σg² partials, the clip coefficient as a device
  scalar, and an update that also emits the bf16 copy gathered by the next forward pass.

Optimizer state dicts keep PyTorch's layout (``state`` + ``param_groups`` with the extra fields
``param_names``, ``sharded``, ``max_grad_norm``, ``max_grad_norm_ratio``) so checkpoints interchange
with the reference.
"""
from __future__ import annotations

import logging
import math
from abc import ABCMeta, abstractmethod
from dataclasses import dataclass, replace
from typing import Any, Dict, List, Optional, Tuple, Union

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.optim.optimizer import Optimizer as OptimizerBase

from .config import OptimizerType, SchedulerConfig, SchedulerType, TrainConfig
from .torch_util import get_default_device, is_distributed

__all__ = [
    "Optimizer",
    "LionW",
    "AdamW",
    "Scheduler",
    "CosWithWarmup",
    "LinearWithWarmup",
    "InvSqrtWithWarmup",
    "MaxScheduler",
    "ConstantScheduler",
    "CosLinearEnvelope",
    "BoltOnWarmupScheduler",
    "ConstantWithWarmupScheduler",
    "build_optimizer",
    "build_scheduler",
    "get_param_groups",
    "fix_optim_state_dict",
    "PARAM_GROUP_FIELDS",
]

log = logging.getLogger(__name__)

PARAM_GROUP_FIELDS = ("sharded", "max_grad_norm", "max_grad_norm_ratio", "param_names")


def _clean(name: str) -> str:
    return name.replace("_fsdp_wrapped_module.", "")


class Optimizer(OptimizerBase):
    """Base class adding distributed gradient clipping and metric collection to a torch optimizer."""

    def __init__(self, *args, record_update_metrics: bool = False, selective_updates: bool = False, **kwargs):
        super().__init__(*args, **kwargs)
        self._record_update_metrics = record_update_metrics
        self._collecting_metrics = False
        self._selective_updates = selective_updates
        self._engine = None  # FlatShardEngine, when parameters are flat-shard views

    # ------------------------------------------------------------------ engine attachment
    def attach_engine(self, engine) -> None:
        """Use fused whole-shard kernels for clipping and the update (parameters must be the engine's views)."""
        self._engine = engine

    def _clean_param_name(self, name: str) -> str:
        return _clean(name)

    def get_state_for_param(self, param: nn.Parameter) -> Dict[str, Optional[torch.Tensor]]:
        del param
        return {}

    def get_post_step_metrics(self, module: nn.Module, process_group: Optional[dist.ProcessGroup] = None) -> Dict[str, torch.Tensor]:
        del module, process_group
        return {}

    # ----------------------------------------------------------------------------- clipping
    @torch.no_grad()
    def clip_grads_and_collect_metrics(
        self,
        global_step: int,
        collect_param_metrics: bool = True,
        process_group: Optional[dist.ProcessGroup] = None,
        device: Optional[torch.device] = None,
    ) -> Dict[str, torch.Tensor]:
        """
        Clip gradients of every group that sets ``max_grad_norm`` (global norm) or ``max_grad_norm_ratio``
        (per parameter, against an EMA of its norm) and return metrics: ``total_grad_norm``, per-parameter
        ``grad/{name}.norm`` and — when ``collect_param_metrics`` — min/max/avg/norm of every parameter,
        gradient and optimizer-state tensor plus ``clipping_rate``.  Norms of sharded parameters are
        summed over ``process_group``.
        """
        self._collecting_metrics = collect_param_metrics
        device = get_default_device() if device is None else device
        if self._engine is not None:
            self._engine.finish_grad_sync()  # gradients of all micro-batches are reduced into the local shards first

        fast = self._fused_clip(global_step, collect_param_metrics, process_group)
        if fast is not None:
            return fast

        names: List[str] = []  # metric prefix per tensor, e.g. "grad/transformer.wte.weight"
        tensors: List[Optional[torch.Tensor]] = []
        for group in self.param_groups:
            for name, p in zip(group["param_names"], group["params"]):
                name = _clean(name)
                names.append(f"grad/{name}")
                tensors.append(p.grad)
                if collect_param_metrics:
                    state = self.get_state_for_param(p)
                    names.append(f"param/{name}")
                    tensors.append(p)
                    for key in sorted(state):
                        names.append(f"{key}/{name}")
                        tensors.append(state[key])

        present = [i for i, t in enumerate(tensors) if t is not None and t.numel() > 0]
        n = len(tensors)
        sq = torch.zeros(n, dtype=torch.float32, device=device)
        if present:
            norms = torch._foreach_norm([tensors[i].detach().float() if tensors[i].dtype != torch.float32 else tensors[i].detach() for i in present], 2)  # type: ignore[union-attr]
            sq[present] = torch.stack([v.to(device) for v in norms]).float() ** 2
        mins = maxs = sums = numels = None
        if collect_param_metrics:
            mins = torch.full((n,), float("inf"), dtype=torch.float32, device=device)
            maxs = torch.zeros(n, dtype=torch.float32, device=device)
            sums = torch.zeros(n, dtype=torch.float32, device=device)
            numels = torch.zeros(n, dtype=torch.float32, device=device)
            for i in present:
                t = tensors[i].detach()  # type: ignore[union-attr]
                a = t.abs()
                mins[i], maxs[i], sums[i], numels[i] = a.min().float(), a.max().float(), t.sum().float(), float(t.numel())

        sharded = any(g.get("sharded", False) for g in self.param_groups)
        if is_distributed() and sharded:
            dst = 0 if process_group is None else dist.get_global_rank(process_group, 0)
            if collect_param_metrics:
                dist.reduce(mins, dst, op=dist.ReduceOp.MIN, group=process_group)
                dist.reduce(maxs, dst, op=dist.ReduceOp.MAX, group=process_group)
                packed = torch.stack([sums, sq, numels])  # type: ignore[list-item]
                dist.all_reduce(packed, op=dist.ReduceOp.SUM, group=process_group)
                sums, sq, numels = packed[0], packed[1], packed[2]
            else:
                dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=process_group)

        is_grad = torch.tensor([nm.startswith("grad/") for nm in names], device=device)
        total_grad_norm = (sq * is_grad).sum().sqrt()
        per_norm = sq.sqrt()

        metrics: Dict[str, torch.Tensor] = {}
        if collect_param_metrics:
            avgs = sums / numels  # type: ignore[operator]
            for i, nm in enumerate(names):
                metrics[f"{nm}.min"] = mins[i]  # type: ignore[index]
            for i, nm in enumerate(names):
                metrics[f"{nm}.max"] = maxs[i]  # type: ignore[index]
            for i, nm in enumerate(names):
                metrics[f"{nm}.avg"] = avgs[i]
        for i, nm in enumerate(names):
            metrics[f"{nm}.norm"] = per_norm[i]
        metrics["total_grad_norm"] = total_grad_norm

        clipped = eligible = 0
        for group in self.param_groups:
            ratio, fixed = group.get("max_grad_norm_ratio"), group.get("max_grad_norm")
            if ratio is not None:
                c = self._do_adaptive_clipping(group, ratio, global_step, metrics, collect_param_metrics)
            elif fixed is not None:
                c = self._do_global_fixed_clipping(group, fixed, metrics, collect_param_metrics)
            else:
                continue
            eligible += len(group["params"])
            clipped += c or 0
        if collect_param_metrics:
            metrics["clipping_rate"] = torch.tensor(clipped / eligible if eligible else 0.0, device="cpu")
        return metrics

    def _fused_clip(self, global_step, collect_param_metrics, process_group) -> Optional[Dict[str, torch.Tensor]]:
        """Whole-shard path: only total norm + fixed global clipping, no per-parameter metrics."""
        eng = self._engine
        if eng is None or collect_param_metrics or not eng.fused_optimizer_ready:
            return None
        limits = {g.get("max_grad_norm") for g in self.param_groups}
        if any(g.get("max_grad_norm_ratio") is not None for g in self.param_groups) or len(limits) != 1:
            return None
        max_norm = limits.pop()
        total = eng.fused_grad_norm_and_clip_coef(max_norm, process_group)
        self._pending_gscale = eng.clip_coef if max_norm is not None else None
        return {"total_grad_norm": total}

    @torch.no_grad()
    def _do_adaptive_clipping(
        self, group: Dict[str, Any], max_norm_ratio: float, global_step: int, all_metrics: Dict[str, torch.Tensor],
        collect_param_metrics: bool = True, device: Optional[torch.device] = None,
    ) -> Optional[int]:
        """Clip each parameter's gradient to ``max_norm_ratio ×`` the EMA of its own past norms."""
        device = get_default_device() if device is None else device
        n_clipped = 0
        beta = max(group["betas"])
        for name, p in zip(group["param_names"], group["params"]):
            name = _clean(name)
            grad_norm = all_metrics.get(f"grad/{name}.norm")
            if grad_norm is None:
                continue
            state = self.state[p]
            ema = state.get("grad_norm_exp_avg")
            if ema is None:
                ema = grad_norm.clone().to(device)
                if global_step > 1:  # the very first norm is often an outlier; don't seed the EMA with it
                    state["grad_norm_exp_avg"] = ema
            coef = torch.clamp(max_norm_ratio * ema / (grad_norm + 1e-6), max=1.0)
            if p.grad is not None:
                p.grad.detach().mul_(coef.to(p.grad.device, p.grad.dtype))
            ema.lerp_((grad_norm * coef).to(ema.device), 1 - beta)
            if collect_param_metrics:
                n_clipped += int(coef < 1.0)
                all_metrics[f"grad_norm_exp_avg/{name}"] = ema
        return n_clipped if collect_param_metrics else None

    @torch.no_grad()
    def _do_global_fixed_clipping(
        self, group: Dict[str, Any], max_norm: float, all_metrics: Dict[str, torch.Tensor],
        collect_param_metrics: bool = True, device: Optional[torch.device] = None,
    ) -> Optional[int]:
        """Scale every gradient of the group by ``min(1, max_norm / (total_norm + 1e-6))``."""
        device = get_default_device() if device is None else device
        coef = torch.clamp(max_norm / (all_metrics["total_grad_norm"].to(device) + 1e-6), max=1.0)
        grads = [p.grad for p in group["params"] if p.grad is not None and p.grad.numel() > 0]
        if grads:
            by_dev: Dict[Tuple[torch.device, torch.dtype], List[torch.Tensor]] = {}
            for g in grads:
                by_dev.setdefault((g.device, g.dtype), []).append(g.detach())
            for (dev, dt), gs in by_dev.items():
                torch._foreach_mul_(gs, coef.to(dev, dt))
        if collect_param_metrics:
            return len(group["params"]) if bool(coef < 1.0) else None
        return None


class LionW(Optimizer):
    """Lion with decoupled weight decay: ``p ← p(1 − lr·wd) − lr·sign(β₁m + (1−β₁)g)``, ``m ← β₂m + (1−β₂)g``."""

    def __init__(
        self,
        params,
        lr: float = 1e-4,
        betas: Tuple[float, float] = (0.9, 0.99),
        weight_decay: float = 0.0,
        record_update_metrics: bool = False,
        selective_updates: bool = False,
        device: Optional[torch.device] = None,
    ):
        assert lr > 0.0
        assert all(0.0 <= b <= 1.0 for b in betas)
        super().__init__(
            params, dict(lr=lr, betas=betas, weight_decay=weight_decay),
            record_update_metrics=record_update_metrics, selective_updates=selective_updates,
        )
        for group in self.param_groups:
            group["initial_lr"] = group["lr"]
        self._device = device
        self._cos_sim_terms: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None

    def get_state_for_param(self, param: nn.Parameter) -> Dict[str, Optional[torch.Tensor]]:
        return {"exp_avg": self.state[param].get("exp_avg")}

    def get_post_step_metrics(self, module: nn.Module, process_group: Optional[dist.ProcessGroup] = None) -> Dict[str, torch.Tensor]:
        """``update_cos_sim``: cosine between the raw update and its sign, over all (sharded) parameters."""
        if self._cos_sim_terms is None:
            return {}
        dot, upd_sq, sgn_sq = self._cos_sim_terms
        self._cos_sim_terms = None
        if is_distributed() and any(g.get("sharded", False) for g in self.param_groups):
            packed = torch.stack([dot, upd_sq, sgn_sq])
            dist.reduce(packed, 0 if process_group is None else dist.get_global_rank(process_group, 0), group=process_group)
            dot, upd_sq, sgn_sq = packed
        denom = torch.clamp(upd_sq.sqrt() * sgn_sq.sqrt(), min=1e-8)
        return {"update_cos_sim": dot / denom}

    @torch.no_grad()
    def step(self, closure=None) -> None:
        if closure is not None:
            with torch.enable_grad():
                closure()
        eng = self._engine
        want_metrics = self._collecting_metrics and self._record_update_metrics
        if eng is not None and eng.fused_optimizer_ready and not want_metrics and not self._selective_updates:
            eng.fused_optimizer_step(self, "lionw", getattr(self, "_pending_gscale", None))
            self._pending_gscale = None
            return
        if eng is not None:
            eng.finish_grad_sync()
        dev = self._device or get_default_device()
        dot = torch.zeros((), dtype=torch.float32, device=dev)
        upd_sq = torch.zeros((), dtype=torch.float32, device=dev)
        sgn_sq = torch.zeros((), dtype=torch.float32, device=dev)
        for group in self.param_groups:
            lr, wd = group["lr"], group["weight_decay"]
            beta1, beta2 = group["betas"]
            for p in group["params"]:
                grad = p.grad
                if grad is None or p.numel() == 0:
                    continue
                state = self.state[p]
                if "exp_avg" not in state:
                    state["exp_avg"] = torch.zeros_like(p)
                m = state["exp_avg"]
                mask: Union[torch.Tensor, int] = (grad != 0) if self._selective_updates else 1
                p.mul_(1 - mask * (lr * wd))
                update = m * beta1 + grad * (1 - beta1)
                if isinstance(mask, torch.Tensor):
                    update.mul_(mask)
                signed = torch.sign(update)
                p.add_(signed, alpha=-lr)
                m.mul_(1 - mask * (1 - beta2)).add_(grad, alpha=1 - beta2)
                if want_metrics:
                    dot += (update.float() * signed.float()).sum().to(dev)
                    upd_sq += update.float().square().sum().to(dev)
                    sgn_sq += signed.float().square().sum().to(dev)
        if want_metrics:
            self._cos_sim_terms = (dot, upd_sq, sgn_sq)
        if eng is not None:
            eng.after_unfused_optimizer_step()


class AdamW(Optimizer):
    """AdamW (decoupled weight decay), numerically the same update as ``torch.optim.AdamW``.

    Options: ``selective_updates`` freezes parameters and moments where the gradient is exactly zero;
    ``record_update_metrics`` keeps the norm and max of every parameter's update for logging.
    """

    def __init__(
        self,
        params,
        lr: float = 1e-3,
        betas: Tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
        amsgrad: bool = False,
        record_update_metrics: bool = False,
        selective_updates: bool = False,
    ):
        defaults = dict(
            lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=amsgrad,
            foreach=None, maximize=False, capturable=False, differentiable=False, fused=None,
        )
        super().__init__(params, defaults, record_update_metrics=record_update_metrics, selective_updates=selective_updates)
        self._step_size_param_names: Optional[List[str]] = None
        self._step_size_norms: Optional[List[torch.Tensor]] = None
        self._step_size_maxs: Optional[List[torch.Tensor]] = None

    def get_state_for_param(self, param: nn.Parameter) -> Dict[str, Optional[torch.Tensor]]:
        return {key: self.state[param].get(key) for key in ("exp_avg", "exp_avg_sq")}

    def _init_state(self, p: torch.Tensor, amsgrad: bool) -> Dict[str, Any]:
        state = self.state[p]
        if len(state) == 0 or "exp_avg" not in state:
            state.setdefault("step", torch.tensor(0.0, dtype=torch.float32))
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            if amsgrad:
                state["max_exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        return state

    @torch.no_grad()
    def step(self, closure=None) -> None:
        if closure is not None:
            with torch.enable_grad():
                closure()
        eng = self._engine
        want_metrics = self._record_update_metrics and self._collecting_metrics
        if eng is not None and eng.fused_optimizer_ready and not want_metrics and not self._selective_updates:
            eng.fused_optimizer_step(self, "adamw", getattr(self, "_pending_gscale", None))
            self._pending_gscale = None
            return
        if eng is not None:
            eng.finish_grad_sync()
        dev = get_default_device()
        names: List[str] = []
        norms: List[torch.Tensor] = []
        maxs: List[torch.Tensor] = []
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            lr, wd, eps, amsgrad = group["lr"], group["weight_decay"], group["eps"], group["amsgrad"]
            for name, p in zip(group.get("param_names", [""] * len(group["params"])), group["params"]):
                names.append(_clean(name))
                grad = p.grad
                if grad is None or p.numel() == 0:
                    norms.append(torch.zeros(1, device=dev))
                    maxs.append(torch.zeros(1, device=dev))
                    continue
                state = self._init_state(p, amsgrad)
                m, v, step_t = state["exp_avg"], state["exp_avg_sq"], state["step"]
                step_t += 1
                step = step_t.item()
                mask: Union[torch.Tensor, int] = (grad != 0) if self._selective_updates else 1
                p.mul_(1 - mask * (lr * wd))
                m.lerp_(grad, mask * (1 - beta1)) if isinstance(mask, torch.Tensor) else m.lerp_(grad, 1 - beta1)
                v.mul_(1 - mask * (1 - beta2)).addcmul_(grad, grad, value=1 - beta2)
                bias1, bias2 = 1 - beta1**step, 1 - beta2**step
                if amsgrad:
                    torch.maximum(state["max_exp_avg_sq"], v, out=state["max_exp_avg_sq"])
                    denom = (state["max_exp_avg_sq"].sqrt() / math.sqrt(bias2)).add_(eps)
                else:
                    denom = (v.sqrt() / math.sqrt(bias2)).add_(eps)
                update = -(lr / bias1) * torch.div(m, denom)
                if isinstance(mask, torch.Tensor):
                    update.mul_(mask)
                p.add_(update)
                if want_metrics:
                    norms.append(torch.linalg.vector_norm(update, 2.0, dtype=torch.float32).unsqueeze(0))
                    maxs.append(update.abs().max().unsqueeze(0))
        if want_metrics:
            self._step_size_param_names, self._step_size_norms, self._step_size_maxs = names, norms, maxs
        if eng is not None:
            eng.after_unfused_optimizer_step()

    def get_post_step_metrics(self, module: nn.Module, process_group: Optional[dist.ProcessGroup] = None) -> Dict[str, torch.Tensor]:
        if not (self._record_update_metrics and self._collecting_metrics) or self._step_size_norms is None:
            return {}
        dev = get_default_device()
        names, norms, maxs = self._step_size_param_names, self._step_size_norms, self._step_size_maxs
        assert names is not None and maxs is not None
        sq = torch.cat(norms).to(dev) ** 2.0
        mx = torch.cat(maxs).to(dev)
        if is_distributed() and any(g.get("sharded", False) for g in self.param_groups):
            dst = 0 if process_group is None else dist.get_global_rank(process_group, 0)
            dist.reduce(sq, dst, op=dist.ReduceOp.SUM, group=process_group)
            dist.reduce(mx, dst, op=dist.ReduceOp.MAX, group=process_group)
        metrics = {}
        for i, name in enumerate(names):
            metrics[f"step/{name}.norm"] = sq[i].sqrt()
            metrics[f"step/{name}.max"] = mx[i]
        self._step_size_param_names = self._step_size_norms = self._step_size_maxs = None
        return metrics


# ------------------------------------------------------------------------------------- schedulers


@dataclass
class Scheduler(metaclass=ABCMeta):
    """Maps a step (or token count, when the trainer runs the schedule in token units) to an LR."""

    grad_clip_warmup_steps: Optional[int]
    grad_clip_warmup_factor: Optional[float]
    warmup_min_lr: Optional[float]

    @abstractmethod
    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        raise NotImplementedError

    def _get_max_grad_norm_coeff(self, initial_value: Optional[float], step: int, max_steps: int) -> Optional[float]:
        del max_steps
        if initial_value is None:
            return None
        warming = (
            self.grad_clip_warmup_steps is not None
            and self.grad_clip_warmup_factor is not None
            and step <= self.grad_clip_warmup_steps
        )
        return self.grad_clip_warmup_factor * initial_value if warming else initial_value  # type: ignore[operator]

    def get_max_grad_norm(self, initial_max_grad_norm: Optional[float], step: int, max_steps: int) -> Optional[float]:
        return self._get_max_grad_norm_coeff(initial_max_grad_norm, step, max_steps)

    def get_max_grad_norm_ratio(self, initial_max_grad_norm_ratio: Optional[float], step: int, max_steps: int) -> Optional[float]:
        return self._get_max_grad_norm_coeff(initial_max_grad_norm_ratio, step, max_steps)

    def _linear_warmup(self, initial_lr: float, step: int, warmup_steps: int = 2000) -> float:
        floor = self.warmup_min_lr if self.warmup_min_lr is not None else initial_lr * 0.10
        assert 0 <= floor < initial_lr
        return floor + (initial_lr - floor) * min(step, warmup_steps) / warmup_steps


def _decay_progress(step: int, warmup: int, horizon: int) -> float:
    return (step - warmup) / (horizon - warmup)


@dataclass
class CosWithWarmup(Scheduler):
    warmup_steps: int
    alpha_f: float = 0.1
    t_max: Optional[int] = None

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        horizon = max_steps if self.t_max is None else self.t_max
        floor = initial_lr * self.alpha_f
        if step < self.warmup_steps:
            return self._linear_warmup(initial_lr, step, self.warmup_steps)
        if step >= horizon:
            return floor
        x = _decay_progress(step, self.warmup_steps, horizon)
        return floor + (initial_lr - floor) * (1 + math.cos(math.pi * x)) / 2


@dataclass
class LinearWithWarmup(Scheduler):
    warmup_steps: int
    alpha_f: float = 0.1
    t_max: Optional[int] = None

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        horizon = max_steps if self.t_max is None else self.t_max
        floor = initial_lr * self.alpha_f
        if step < self.warmup_steps:
            return self._linear_warmup(initial_lr, step, self.warmup_steps)
        if step >= horizon:
            return floor
        return initial_lr - (initial_lr - floor) * _decay_progress(step, self.warmup_steps, horizon)


@dataclass
class InvSqrtWithWarmup(Scheduler):
    warmup_steps: int

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        del max_steps
        if step < self.warmup_steps:
            return self._linear_warmup(initial_lr, step, self.warmup_steps)
        return initial_lr * math.sqrt(self.warmup_steps / max(self.warmup_steps, step))


@dataclass
class MaxScheduler(Scheduler):
    sched1: Scheduler
    sched2: Scheduler

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        return max(self.sched1.get_lr(initial_lr, step, max_steps), self.sched2.get_lr(initial_lr, step, max_steps))


@dataclass
class BoltOnWarmupScheduler(Scheduler):
    """A fresh linear warm-up from 0 that meets the wrapped schedule at ``warmup_end`` (used after an
    optimizer-state reset)."""

    inner: Scheduler
    warmup_start: int
    warmup_end: int

    @classmethod
    def wrap(cls, scheduler: Scheduler, warmup_start: int, warmup_end: int) -> "BoltOnWarmupScheduler":
        return cls(
            grad_clip_warmup_steps=None, grad_clip_warmup_factor=None, warmup_min_lr=None,
            inner=scheduler, warmup_start=warmup_start, warmup_end=warmup_end,
        )

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        if step < self.warmup_start:
            return 0.0
        if step < self.warmup_end:
            target = self.inner.get_lr(initial_lr, self.warmup_end, max_steps)
            return target * (step - self.warmup_start) / (self.warmup_end - self.warmup_start)
        return self.inner.get_lr(initial_lr, step, max_steps)

    def _get_max_grad_norm_coeff(self, initial_value: Optional[float], step: int, max_steps: int) -> Optional[float]:
        return self.inner._get_max_grad_norm_coeff(initial_value, step, max_steps)


@dataclass
class ConstantScheduler(Scheduler):
    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        del step, max_steps
        return initial_lr


@dataclass
class CosLinearEnvelope(Scheduler):
    """Cosine decay multiplied by a linear ramp to zero (annealing)."""

    warmup_steps: int
    alpha_f: float = 0.1
    t_max: Optional[int] = None

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        horizon = max_steps if self.t_max is None else self.t_max
        floor = initial_lr * self.alpha_f
        if step < self.warmup_steps:
            return self._linear_warmup(initial_lr, step, self.warmup_steps)
        if step >= horizon:
            return floor
        x = _decay_progress(step, self.warmup_steps, horizon)
        return floor + (1 - x) * (initial_lr - floor) * (1 + math.cos(math.pi * x)) / 2


@dataclass
class ConstantWithWarmupScheduler(Scheduler):
    warmup_steps: int

    def get_lr(self, initial_lr: float, step: int, max_steps: int) -> float:
        del max_steps
        if step < self.warmup_steps:
            return self._linear_warmup(initial_lr, step, self.warmup_steps)
        return initial_lr


# --------------------------------------------------------------------------------------- builders


def _is_sharded_model(model: nn.Module) -> bool:
    return bool(getattr(model, "is_flat_sharded", False))


def get_param_groups(cfg: TrainConfig, model: nn.Module) -> List[Dict[str, Any]]:
    """Split parameters into a weight-decay group and a no-decay group, each sorted by name.

    Linear weights always decay; norm weights and all biases decay only with ``decay_norm_and_bias``;
    embeddings only with ``decay_embeddings``.
    """
    from .models.layers import LayerNormBase

    named = model.named_parameters_for_optimizer() if hasattr(model, "named_parameters_for_optimizer") else None
    kinds: Dict[str, str] = {}
    module_root = getattr(model, "module", model) if named is not None else model
    for mn, m in module_root.named_modules():
        for pn, p in m.named_parameters(recurse=False):
            if named is None and not p.requires_grad:
                continue
            fpn = f"{mn}.{pn}" if mn else pn
            if pn.endswith("bias"):
                kinds[fpn] = "norm_or_bias"
            elif pn.endswith("weight") and isinstance(m, nn.Linear):
                kinds[fpn] = "linear"
            elif pn.endswith("weight") and isinstance(m, (LayerNormBase, nn.LayerNorm)):
                kinds[fpn] = "norm_or_bias"
            elif pn.endswith("weight") and isinstance(m, nn.Embedding):
                kinds[fpn] = "embedding"
    all_params: Dict[str, torch.Tensor] = dict(named) if named is not None else {
        n: p for n, p in module_root.named_parameters() if p.requires_grad
    }
    # tied weights appear under one name only in named_parameters(); restrict kinds to those names
    missing = set(all_params) - set(kinds)
    assert not missing, f"parameters {missing} were not separated into either decay/no_decay set!"
    decay, no_decay = [], []
    for name in all_params:
        kind = kinds[name]
        decays = kind == "linear" or (kind == "norm_or_bias" and cfg.optimizer.decay_norm_and_bias) or (
            kind == "embedding" and cfg.optimizer.decay_embeddings
        )
        (decay if decays else no_decay).append(name)
    shared = {
        "sharded": _is_sharded_model(model),
        "max_grad_norm": cfg.max_grad_norm,
        "max_grad_norm_ratio": cfg.max_grad_norm_ratio,
    }
    groups: List[Dict[str, Any]] = []
    if decay:
        names = sorted(decay)
        groups.append({"params": [all_params[n] for n in names], "param_names": names, **shared})
    if no_decay:
        names = sorted(no_decay)
        groups.append({"params": [all_params[n] for n in names], "param_names": names, "weight_decay": 0.0, **shared})
    return groups


def fix_optim_state_dict(optimizer: Optimizer, state_dict: Dict[str, Any]) -> Dict[str, Any]:
    """Upgrade an old single-group optimizer state dict to the decay / no-decay pair and refresh the
    bookkeeping fields from the live optimizer."""
    if len(state_dict["param_groups"]) == 1 and len(optimizer.param_groups) == 2:
        assert optimizer.param_groups[1]["weight_decay"] == 0.0
        live = optimizer.state_dict()["param_groups"]
        base = {k: v for k, v in state_dict["param_groups"][0].items() if k != "params"}
        state_dict["param_groups"] = [
            {**base, "params": live[0]["params"]},
            {**base, "weight_decay": 0.0, "params": live[1]["params"]},
        ]
    assert len(optimizer.param_groups) == len(state_dict["param_groups"])
    for group, sd_group in zip(optimizer.param_groups, state_dict["param_groups"]):
        for key in PARAM_GROUP_FIELDS:
            sd_group[key] = group[key]
    return state_dict


def build_optimizer(cfg: TrainConfig, model: nn.Module) -> Optimizer:
    groups = get_param_groups(cfg, model)
    log.info("Constructing optimizer with %d param groups", len(groups))
    common = dict(
        lr=cfg.optimizer.learning_rate,
        betas=tuple(cfg.optimizer.betas),
        weight_decay=cfg.optimizer.weight_decay,
        record_update_metrics=cfg.optimizer.record_update_metrics,
        selective_updates=cfg.optimizer.selective_updates,
    )
    if cfg.optimizer.name == OptimizerType.lionw:
        opt: Optimizer = LionW(groups, **common)
    elif cfg.optimizer.name == OptimizerType.adamw:
        opt = AdamW(groups, eps=cfg.optimizer.eps, **common)
    else:
        raise NotImplementedError(cfg.optimizer.name)
    if hasattr(model, "engine"):
        opt.attach_engine(model.engine)
    return opt


def build_scheduler(cfg: TrainConfig, sched_cfg: Optional[SchedulerConfig] = None) -> Scheduler:
    sc = sched_cfg if sched_cfg is not None else cfg.scheduler
    base = dict(
        grad_clip_warmup_steps=None if sc.grad_clip_warmup_steps is None else int(sc.grad_clip_warmup_steps),
        grad_clip_warmup_factor=sc.grad_clip_warmup_factor,
        warmup_min_lr=sc.warmup_min_lr,
    )
    warm = dict(warmup_steps=int(sc.t_warmup))
    decay = dict(alpha_f=sc.alpha_f, t_max=None if sc.t_max is None else int(sc.t_max))
    if sc.name == SchedulerType.cosine_with_warmup:
        return CosWithWarmup(**base, **warm, **decay)
    if sc.name == SchedulerType.linear_with_warmup:
        return LinearWithWarmup(**base, **warm, **decay)
    if sc.name == SchedulerType.inverse_sqrt_with_warmup:
        return InvSqrtWithWarmup(**base, **warm)
    if sc.name == SchedulerType.max_scheduler:
        return MaxScheduler(
            **base,
            sched1=build_scheduler(cfg, replace(sc, name=SchedulerType.cosine_with_warmup)),
            sched2=build_scheduler(cfg, replace(sc, name=SchedulerType.inverse_sqrt_with_warmup)),
        )
    if sc.name == SchedulerType.constant:
        return ConstantScheduler(**base)
    if sc.name == SchedulerType.cosine_linear_envelope:
        return CosLinearEnvelope(**base, **warm, **decay)
    if sc.name == SchedulerType.constant_with_warmup:
        return ConstantWithWarmupScheduler(**base, **warm)
    raise NotImplementedError(sc.name)
