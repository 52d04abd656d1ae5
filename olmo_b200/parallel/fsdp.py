"""
Flat-shard data-parallel engine: this framework's replacement for ``torch`` FSDP1 / DDP wrapping
(reference: ``scripts/train.py:154-230``; strategies in ``olmo/config.py:741-866``).

Layout
------
The model is partitioned into *units* (per block, ``wte``, ``ff_out``, root — the same partitions the
reference's wrap policies produce).  Each unit's parameters are laid end to end, 128-byte aligned, in one
flat buffer that is padded and cut into ``shard_world`` equal shards.  A rank holds, per unit,

* ``master``  fp32 shard of the parameters                      (what the optimizer updates)
* ``grad``    fp32 shard of the accumulated, reduced gradient
* ``lowp``    compute-dtype copy of the shard                   (what peers gather from)
* ``full``    compute-dtype copy of the whole unit              (module parameters are views into it)
* ``gfull``   fp32 gradient of the whole unit before reduction  (aliases ``grad`` when nothing is sharded)

The optimizer sees one ``nn.Parameter`` per (parameter ∩ shard) named by the original FQN, exactly the view
``use_orig_params=True`` gives in FSDP1, so param groups, metrics and checkpoints keep their meaning.

Execution
---------
``fused``     CUDA + bf16 + a configuration the kernels cover: forward and backward are explicit kernel
              sequences (:mod:`olmo_b200.ops.fused_block`), weight gradients accumulate in fp32 straight from the
              GEMM epilogue, the optimizer runs as whole-shard kernels, and — with more than one GPU —
              gathers/reductions go through peer memory (:mod:`olmo_b200.parallel.peer`).
``portable``  anything else (CPU/Gloo ranks, fp32, ALiBi, llama blocks, …): autograd on the gathered
              parameters plus ``torch.distributed`` collectives.  Same layout, same checkpoints.

Strategy mapping: ``FULL_SHARD``/``SHARD_GRAD_OP`` shard over all ranks, ``HYBRID_SHARD``/``_HYBRID_SHARD_ZERO2``
shard inside a replica group and all-reduce across groups, ``NO_SHARD`` and ``ddp`` replicate.  With 180 GB per
device the gathered compute copy of every unit stays resident between uses and gradients of all micro-batches are
accumulated locally in fp32, so each optimizer step pays one gather and one reduction per unit instead of one per
micro-batch; ``OLMO_B200_RESHARD=1`` restores the gather-per-use / reduce-per-micro-batch schedule.
"""
from __future__ import annotations

import logging
import math
import os
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, Iterator, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from ..config import (
    ActivationCheckpointingStrategy,
    DistributedStrategy,
    ShardingStrategy,
    TrainConfig,
)
from ..exceptions import OLMoConfigurationError
from ..models.blocks import OLMoBlock, should_checkpoint_block
from ..models.olmo import OLMo, OLMoOutput
from ..torch_util import get_global_rank, get_world_size, is_distributed, nvtx_range

__all__ = ["FlatShardEngine", "ShardedModel", "Unit", "ParamSlot", "build_sharded_model"]

log = logging.getLogger(__name__)

ALIGN = 64  # elements; keeps every parameter 128-byte aligned in bf16 and 256-byte aligned in fp32


@dataclass
class ParamSlot:
    name: str  # fully-qualified parameter name inside the OLMo module
    shape: torch.Size
    numel: int
    offset: int  # start inside the unit's flat buffer
    owner: nn.Module
    attr: str


@dataclass
class Unit:
    name: str
    index: int
    slots: List[ParamSlot]
    numel: int  # padded flat length (multiple of shard_world * 1024)
    shard_size: int
    master: torch.Tensor = field(default=None, repr=False)  # type: ignore[assignment]
    grad: torch.Tensor = field(default=None, repr=False)  # type: ignore[assignment]
    lowp: torch.Tensor = field(default=None, repr=False)  # type: ignore[assignment]
    full: torch.Tensor = field(default=None, repr=False)  # type: ignore[assignment]
    gfull: torch.Tensor = field(default=None, repr=False)  # type: ignore[assignment]
    gfull_dirty: Dict[str, bool] = field(default_factory=dict, repr=False)
    state: Dict[str, torch.Tensor] = field(default_factory=dict, repr=False)  # flat optimizer state shards
    seg_end: Optional[torch.Tensor] = field(default=None, repr=False)
    seg_wd: Optional[torch.Tensor] = field(default=None, repr=False)
    seg_lr: Optional[torch.Tensor] = field(default=None, repr=False)
    seg_meta: List[Tuple[int, int]] = field(default_factory=list, repr=False)  # (group index, end offset in shard)

    def slot(self, name: str) -> ParamSlot:
        for s in self.slots:
            if s.name == name:
                return s
        raise KeyError(name)


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class FlatShardEngine:
    def __init__(
        self,
        model: OLMo,
        cfg: TrainConfig,
        device: torch.device,
        *,
        seed: Optional[int] = None,
        force_portable: bool = False,
    ):
        self.model = model
        self.cfg = cfg
        self.device = device
        self.world = get_world_size()
        self.rank = get_global_rank()
        self._setup_groups()

        strategy = cfg.distributed_strategy
        precision = cfg.precision or "fp32"
        self.compute_dtype = cfg.autocast_precision if precision != "fp32" else torch.float32
        if strategy == DistributedStrategy.fsdp and cfg.fsdp is not None and cfg.fsdp.precision is None:
            self.compute_dtype = torch.float32
        from ..ops import enabled as kernels_enabled
        from ..ops import fused_block

        self.fused = (
            not force_portable
            and device.type == "cuda"
            and kernels_enabled()
            and self.compute_dtype == torch.bfloat16
            and fused_block.config_supported(model.config)
            and not model.config.embedding_layer_norm
            and model.config.embedding_dropout == 0.0
            and model.config.block_group_size >= 1
        )
        self.reshard = os.environ.get("OLMO_B200_RESHARD", "0") not in ("0", "", "false")
        # Keep the rotated q/k and the SwiGLU output of every block for the backward pass instead of recomputing them:
        # "1"/"0" force it, "auto" decides after the first complete step from the memory that is still free.
        keep = os.environ.get("OLMO_B200_KEEP_ACTS", "auto").strip().lower()
        self.keep_recomputable: Optional[bool] = {"1": True, "true": True, "0": False, "false": False}.get(keep)
        self.units: List[Unit] = []
        self._unit_of_param: Dict[str, Tuple[Unit, ParamSlot]] = {}
        self._opt_params: List[Tuple[str, nn.Parameter]] = []
        self._params_stale = True  # `full` buffers need a gather before the next forward
        self._grads_pending = False  # gfull holds unreduced gradients
        self._microbatches_since_reduce = 0
        self._grad_epoch_open = False
        self.fused_optimizer_ready = False
        self.clip_coef: Optional[torch.Tensor] = None
        self._sumsq: Optional[torch.Tensor] = None
        self._norm_out: Optional[torch.Tensor] = None
        self.comm = None
        self._build(seed if seed is not None else cfg.seed)

    # ------------------------------------------------------------------------------- groups
    def _setup_groups(self) -> None:
        cfg = self.cfg
        self.shard_group: Optional[dist.ProcessGroup] = None
        self.replica_group: Optional[dist.ProcessGroup] = None
        world = self.world
        strategy = ShardingStrategy.NO_SHARD
        if cfg.distributed_strategy == DistributedStrategy.fsdp and cfg.fsdp is not None:
            strategy = cfg.fsdp.sharding_strategy
        self.sharding_strategy = strategy
        if world == 1 or strategy == ShardingStrategy.NO_SHARD or cfg.distributed_strategy in (DistributedStrategy.ddp, DistributedStrategy.single):
            self.shard_world, self.shard_rank = 1, 0
            self.num_replicas = world
            return
        if strategy in (ShardingStrategy.HYBRID_SHARD, ShardingStrategy._HYBRID_SHARD_ZERO2):
            replicas = cfg.fsdp.hybrid_sharding_num_model_replicas  # type: ignore[union-attr]
            if replicas is None:
                from ..torch_util import get_local_world_size

                replicas = max(1, world // max(1, get_local_world_size()))
            if replicas <= 0 or world % replicas != 0:
                raise OLMoConfigurationError("fsdp.hybrid_sharding_num_model_replicas must be a positive divisor of world size")
            per = world // replicas
            self.num_replicas = replicas
            self.shard_world, self.shard_rank = per, self.rank % per
            # ranks [g*per, (g+1)*per) form a shard group; ranks with equal (rank % per) form a replica group
            for g in range(replicas):
                grp = dist.new_group(list(range(g * per, (g + 1) * per)))
                if self.rank // per == g:
                    self.shard_group = grp
            for r in range(per):
                grp = dist.new_group(list(range(r, world, per)))
                if self.rank % per == r:
                    self.replica_group = grp
            return
        self.shard_world, self.shard_rank, self.num_replicas = world, self.rank, 1

    @property
    def process_group(self) -> Optional[dist.ProcessGroup]:
        """Group over which per-shard quantities (gradient norms) are summed."""
        return self.shard_group

    @property
    def is_sharded(self) -> bool:
        return self.shard_world > 1

    # -------------------------------------------------------------------------------- build
    def _collect_units(self) -> List[Tuple[str, List[Tuple[str, nn.Parameter, nn.Module, str]]]]:
        wrap = None
        if self.cfg.distributed_strategy == DistributedStrategy.fsdp and self.cfg.fsdp is not None:
            wrap = self.cfg.fsdp.wrapping_strategy
        if wrap is None and self.fused:
            from ..config import FSDPWrapStrategy

            # the fused path works block by block whatever the requested wrapping was
            wrap = FSDPWrapStrategy.by_block_and_size if self.model.config.block_group_size == 1 else FSDPWrapStrategy.by_block_group_and_size
        names = {id(p): n for n, p in self.model.named_parameters()}
        taken: set = set()
        out = []
        for uname, modules in self.model.fsdp_units(wrap):
            entries = []
            for mod in modules:
                for sub in mod.modules():
                    for attr, p in sub.named_parameters(recurse=False):
                        if id(p) in taken or id(p) not in names:
                            continue
                        taken.add(id(p))
                        entries.append((names[id(p)], p, sub, attr))
            if entries:
                out.append((uname, entries))
        return out

    def _build(self, seed: int) -> None:
        model, dev = self.model, self.device
        # 1. materialise and initialise the full model identically on every rank
        if any(p.is_meta for p in model.parameters()):
            model.to_empty(device=dev)
            torch.manual_seed(seed)
            if dev.type == "cuda":
                torch.cuda.manual_seed(seed)
            model.reset_parameters()
        else:
            model.to(dev)
        # 2. flat layout
        sw = self.shard_world
        for index, (uname, entries) in enumerate(self._collect_units()):
            offset = 0
            slots = []
            for name, p, owner, attr in entries:
                slots.append(ParamSlot(name, p.shape, p.numel(), offset, owner, attr))
                offset = _round_up(offset + p.numel(), ALIGN)
            total = _round_up(max(offset, 1), sw * 1024)
            unit = Unit(uname, index, slots, total, total // sw)
            self.units.append(unit)
        # 3. buffers; module parameters become views of `full`
        use_peer = (
            self.is_sharded and dev.type == "cuda" and self.fused
            and os.environ.get("OLMO_B200_FUSED_COMM", "1").strip().lower() not in ("0", "false", "no", "off")
        )
        if use_peer:
            from .peer import PeerComm

            self.comm = PeerComm.create(self)
        for unit in self.units:
            S, P = unit.shard_size, unit.numel
            lo = self.shard_rank * S
            flat = torch.zeros(P, dtype=torch.float32, device=dev)
            for s in unit.slots:
                flat[s.offset : s.offset + s.numel].copy_(getattr(s.owner, s.attr).detach().reshape(-1).float())
            unit.master = flat[lo : lo + S].clone() if sw > 1 else flat
            unit.grad = torch.zeros(S, dtype=torch.float32, device=dev)
            if self.comm is not None:
                unit.full = self.comm.full_view(unit.index, P)
                unit.full.copy_(flat)
                unit.gfull = self.comm.gfull_view(unit.index, P)
            else:
                unit.full = flat.to(self.compute_dtype) if (self.compute_dtype != torch.float32 or sw > 1) else flat.clone()
                unit.gfull = unit.grad if sw == 1 else None  # type: ignore[assignment]
            unit.lowp = unit.full[lo : lo + S] if sw > 1 else unit.full
            for s in unit.slots:
                view = unit.full[s.offset : s.offset + s.numel].view(s.shape)
                param = nn.Parameter(view, requires_grad=not self.fused)
                param._ob_unit = unit  # type: ignore[attr-defined]
                param._ob_slot = s  # type: ignore[attr-defined]
                s.owner._parameters[s.attr] = param
                self._unit_of_param[s.name] = (unit, s)
            del flat
        if dev.type == "cuda":
            torch.cuda.empty_cache()
        # 4. optimizer-facing parameters: one per (parameter ∩ local shard)
        for unit in self.units:
            lo = self.shard_rank * unit.shard_size
            hi = lo + unit.shard_size
            for s in unit.slots:
                a, b = max(s.offset, lo), min(s.offset + s.numel, hi)
                if b > a:
                    data = unit.master[a - lo : b - lo]
                    gview = unit.grad[a - lo : b - lo]
                    if b - a == s.numel:
                        data, gview = data.view(s.shape), gview.view(s.shape)
                else:
                    data = unit.master[0:0]
                    gview = unit.grad[0:0]
                p = nn.Parameter(data, requires_grad=True)
                p.grad = gview
                p._ob_range = (unit.index, a - lo, max(b, a) - lo)  # type: ignore[attr-defined]
                self._opt_params.append((s.name, p))
        self._params_stale = sw > 1  # `full` was filled from the initial weights; only shards differ after a step
        self._params_stale = False
        if self.fused:
            self._setup_fused()
        if self.is_sharded and self.comm is None:
            for unit in self.units:
                unit.gfull = torch.zeros(unit.numel, dtype=torch.float32, device=dev)
        log.info(
            "FlatShardEngine: %d units, %.2fB parameters, shard world %d, replicas %d, %s path",
            len(self.units), sum(s.numel for u in self.units for s in u.slots) / 1e9, self.shard_world, self.num_replicas,
            "fused" if self.fused else "portable",
        )

    # ----------------------------------------------------------------------- optimizer side
    def named_parameters_for_optimizer(self) -> List[Tuple[str, nn.Parameter]]:
        return list(self._opt_params)

    def _setup_fused(self) -> None:
        dev = self.device
        self.clip_coef = torch.ones(1, dtype=torch.float32, device=dev)
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._norm_out = torch.zeros(1, dtype=torch.float32, device=dev)
        self.fused_optimizer_ready = True

    def _ensure_fused_state(self, optim, kind: str) -> None:
        """Flat optimizer-state shards whose per-parameter views live in ``optim.state`` (so state dicts keep
        PyTorch's shape), plus the per-unit (segment end, weight decay, lr) tables."""
        keys = ("exp_avg", "exp_avg_sq") if kind == "adamw" else ("exp_avg",)
        group_of: Dict[int, int] = {}
        for gi, group in enumerate(optim.param_groups):
            for p in group["params"]:
                group_of[id(p)] = gi
        for unit in self.units:
            if all(key in unit.state for key in keys):
                continue
            for key in keys:
                unit.state[key] = torch.zeros(unit.shard_size, dtype=torch.float32, device=self.device)
            unit.seg_meta = []
        for name, p in self._opt_params:
            ui, a, b = p._ob_range  # type: ignore[attr-defined]
            unit = self.units[ui]
            st = optim.state[p]
            for key in keys:
                view = unit.state[key][a:b].view(p.shape)
                if key in st and st[key].data_ptr() != view.data_ptr():
                    view.copy_(st[key])
                st[key] = view
            st.setdefault("step", torch.tensor(0.0, dtype=torch.float32))
        for unit in self.units:
            if unit.seg_meta:
                continue
            segs = []
            for name, p in self._opt_params:
                ui, a, b = p._ob_range  # type: ignore[attr-defined]
                if ui == unit.index and b > a:
                    segs.append((group_of[id(p)], _round_up(b, 1)))
            if not segs:
                segs = [(0, unit.shard_size)]
            segs[-1] = (segs[-1][0], unit.shard_size)  # padding belongs to the last segment (zeros stay zeros)
            unit.seg_meta = segs
            unit.seg_end = torch.tensor([e for _, e in segs], dtype=torch.int64, device=self.device)
            unit.seg_wd = torch.empty(len(segs), dtype=torch.float32, device=self.device)
            unit.seg_lr = torch.empty(len(segs), dtype=torch.float32, device=self.device)
            unit._seg_host = None  # type: ignore[attr-defined]

    def _refresh_segments(self, optim) -> None:
        for unit in self.units:
            host = [(optim.param_groups[g]["weight_decay"], optim.param_groups[g]["lr"]) for g, _ in unit.seg_meta]
            if getattr(unit, "_seg_host", None) != host:
                unit.seg_wd.copy_(torch.tensor([h[0] for h in host], dtype=torch.float32))  # type: ignore[union-attr]
                unit.seg_lr.copy_(torch.tensor([h[1] for h in host], dtype=torch.float32))  # type: ignore[union-attr]
                unit._seg_host = host  # type: ignore[attr-defined]

    def fused_grad_norm_and_clip_coef(self, max_norm: Optional[float], process_group=None) -> torch.Tensor:
        """Σg² over every local shard (one two-stage reduction kernel per unit), summed over the shard group,
        then the clip coefficient as a device scalar.  Returns the total gradient norm (device tensor)."""
        from ..ops import kernels as k

        self.finish_grad_sync()
        comm = self.comm
        if comm is not None and comm.fuse_sumsq and not self.reshard:
            # every shard was written exactly once this step, by reduce-scatter kernels that also summed its squares
            torch.sum(comm.rs_partials, dim=0, keepdim=True, out=self._sumsq)
        else:
            for i, unit in enumerate(self.units):
                k.sumsq(unit.grad, self._sumsq, accumulate=i > 0)
        if self.is_sharded:
            if self.comm is not None:
                self.comm.all_reduce_scalar_(self._sumsq)
            else:
                dist.all_reduce(self._sumsq, group=process_group or self.shard_group)
        k.clip_coef(self._sumsq, float(max_norm) if max_norm is not None else float("inf"), self.clip_coef, self._norm_out)
        return self._norm_out[0].clone()

    def fused_optimizer_step(self, optim, kind: str, gscale: Optional[torch.Tensor]) -> None:
        from ..ops import kernels as k

        self.finish_grad_sync()
        self._ensure_fused_state(optim, kind)
        self._refresh_segments(optim)
        step = None
        for name, p in self._opt_params:
            st = optim.state[p]
            st["step"] += 1
            if step is None:
                step = int(st["step"].item())
        step = step or 1
        for unit in self.units:
            lowp = unit.lowp if unit.lowp.dtype == torch.bfloat16 else None
            g0 = optim.param_groups[0]
            if kind == "adamw":
                b1, b2 = g0["betas"]
                k.adamw_flat(unit.master, unit.grad, unit.state["exp_avg"], unit.state["exp_avg_sq"], lowp,
                             unit.seg_end, unit.seg_wd, unit.seg_lr, b1, b2, g0["eps"], step, gscale)
            else:
                b1, b2 = g0["betas"]
                k.lionw_flat(unit.master, unit.grad, unit.state["exp_avg"], lowp, unit.seg_end, unit.seg_wd, unit.seg_lr, b1, b2, gscale)
            if lowp is None:
                unit.lowp.copy_(unit.master)
        self._params_stale = True
        if self.comm is not None:
            self.comm.publish_params()

    def after_unfused_optimizer_step(self) -> None:
        """Per-parameter optimizers updated ``master`` in place: refresh the compute-dtype shard."""
        for unit in self.units:
            if unit.lowp.data_ptr() != unit.master.data_ptr():
                unit.lowp.copy_(unit.master)
        self._params_stale = True
        if self.comm is not None:
            self.comm.publish_params()

    def zero_grad(self) -> None:
        for unit in self.units:
            unit.grad.zero_()
            unit.gfull_dirty.clear()
            if unit.gfull is not None and unit.gfull.data_ptr() != unit.grad.data_ptr():
                unit.gfull.zero_()
            unit.reduced = False  # type: ignore[attr-defined]
        if self.comm is not None:
            self.comm.rs_partials.zero_()
        self._microbatches_since_reduce = 0
        self._grads_pending = False

    # -------------------------------------------------------------------------- collectives
    def gather_params(self) -> None:
        """Make every ``full`` buffer current (no-op when nothing changed since the last gather)."""
        if not self._params_stale:
            return
        if self.is_sharded:
            if self.comm is not None:
                self.comm.all_gather_units(self.units)
            else:
                for unit in self.units:
                    dist.all_gather_into_tensor(unit.full, unit.lowp.contiguous(), group=self.shard_group) if self._has_agit() else self._all_gather_fallback(unit)
        self._params_stale = False

    def _has_agit(self) -> bool:
        return self.device.type == "cuda"

    def _all_gather_fallback(self, unit: Unit) -> None:
        chunks = [torch.empty_like(unit.lowp) for _ in range(self.shard_world)]
        dist.all_gather(chunks, unit.lowp.contiguous(), group=self.shard_group)
        for r, c in enumerate(chunks):
            unit.full[r * unit.shard_size : (r + 1) * unit.shard_size].copy_(c)

    def finish_grad_sync(self) -> None:
        """Reduce the locally accumulated full-size gradients into the fp32 shards (average over data-parallel ranks)."""
        if not self._grads_pending:
            return
        self._grads_pending = False
        world = self.world
        if not self.fused:
            self._collect_autograd_grads()
        if world == 1:
            return
        if self.comm is not None:
            pending = [u for u in self.units if not getattr(u, "reduced", False)]
            if pending:
                if not self._grad_epoch_open:
                    self.comm.begin_grad_epoch()
                for u in pending:
                    if not getattr(u, "published", False):
                        self.comm.publish_grads(u)
                self.comm.reduce_scatter_units(pending, scale=1.0 / world)
                for u in pending:
                    u.reduced = True  # type: ignore[attr-defined]
            self._grad_epoch_open = False
            for u in self.units:
                u.published = False  # type: ignore[attr-defined]
        else:
            for unit in self.units:
                src = unit.gfull
                if self.is_sharded:
                    lo = self.shard_rank * unit.shard_size
                    if self.device.type == "cuda":
                        out = torch.empty(unit.shard_size, dtype=torch.float32, device=self.device)
                        dist.reduce_scatter_tensor(out, src, group=self.shard_group)
                    else:
                        dist.all_reduce(src, group=self.shard_group)
                        out = src[lo : lo + unit.shard_size]
                    if self.replica_group is not None:
                        out = out.contiguous()
                        dist.all_reduce(out, group=self.replica_group)
                    unit.grad.add_(out, alpha=1.0 / world)
                    src.zero_()
                else:
                    dist.all_reduce(unit.grad)
                    unit.grad.div_(world)
            for unit in self.units:
                unit.gfull_dirty.clear()

    def _collect_autograd_grads(self) -> None:
        for unit in self.units:
            for s in unit.slots:
                p = getattr(s.owner, s.attr)
                if p.grad is not None:
                    unit.gfull[s.offset : s.offset + s.numel].add_(p.grad.reshape(-1).float())
                    p.grad = None

    def note_microbatch_backward(self) -> None:
        """Called after each micro-batch's backward pass."""
        self._grads_pending = True
        self._microbatches_since_reduce += 1
        if not self.fused:
            self._collect_autograd_grads()
        if self.reshard:
            self.finish_grad_sync()

    # ----------------------------------------------------------------- fused forward/backward
    def _weights_of(self, block: OLMoBlock) -> Dict[str, Optional[torch.Tensor]]:
        def w(mod, attr="weight"):
            return None if mod is None else getattr(mod, attr, None)

        return {
            "att_proj": block.att_proj.weight, "attn_out": block.attn_out.weight,
            "ff_proj": block.ff_proj.weight, "ff_out": block.ff_out.weight,
            "attn_norm": w(block.attn_norm), "ff_norm": w(block.ff_norm),
            "q_norm": w(block.q_norm), "k_norm": w(block.k_norm),
        }

    def grad_view(self, param: nn.Parameter) -> Tuple[torch.Tensor, Unit, ParamSlot]:
        unit: Unit = param._ob_unit  # type: ignore[attr-defined]
        slot: ParamSlot = param._ob_slot  # type: ignore[attr-defined]
        if unit.gfull is None:
            raise RuntimeError("gradient buffer of unit %s is not allocated" % unit.name)
        return unit.gfull[slot.offset : slot.offset + slot.numel].view(slot.shape), unit, slot

    def matrix_grad(self, param: nn.Parameter, dy: torch.Tensor, x: torch.Tensor) -> None:
        """``grad(param) += dyᵀ·x`` in fp32 from the GEMM epilogue (first write after a zero is a plain store)."""
        from ..ops import kernels as k

        g, unit, slot = self.grad_view(param)
        k.gemm(dy, x, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=g)

    def vector_grad(self, param: nn.Parameter) -> torch.Tensor:
        return self.grad_view(param)[0]

    def _unit_of_module_param(self, param: nn.Parameter) -> Unit:
        return param._ob_unit  # type: ignore[attr-defined]

    def _forward_unit_order(self) -> List[Unit]:
        """Units in the order the forward pass first touches them."""
        t = self.model.transformer
        seq = [t.wte.weight] + [b.att_proj.weight for b in self.model.all_blocks()] + [t.ln_f.weight]
        if not self.model.config.weight_tying:
            seq.append(t.ff_out.weight)
        order: List[Unit] = []
        for p in seq:
            if p is None:
                continue
            u = self._unit_of_module_param(p)
            if all(u is not o for o in order):
                order.append(u)
        for u in self.units:
            if all(u is not o for o in order):
                order.append(u)
        return order

    def _unit_final_points(self) -> Dict[int, int]:
        """For the backward pass: unit index -> the block index after whose backward the unit's gradients are final
        (``n_blocks`` = right after the head and final norm, ``-1`` = after the embedding gradient)."""
        blocks = self.model.all_blocks()
        final: Dict[int, int] = {}
        t = self.model.transformer
        head = t.wte.weight if self.model.config.weight_tying else t.ff_out.weight
        for p in (head, t.ln_f.weight):
            if p is not None:
                final[self._unit_of_module_param(p).index] = len(blocks)
        for i in range(len(blocks) - 1, -1, -1):
            final[self._unit_of_module_param(blocks[i].att_proj.weight).index] = i
        final[self._unit_of_module_param(t.wte.weight).index] = -1
        for u in self.units:
            final.setdefault(u.index, -1)
        return final

    def train_microbatch(
        self,
        input_ids: torch.Tensor,
        labels: torch.Tensor,
        loss_divisor: float,
        z_mult: float = 0.0,
        ac_strategy: Optional[ActivationCheckpointingStrategy] = None,
        is_last: bool = True,
        doc_start: Optional[torch.Tensor] = None,
    ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Forward + backward of one micro-batch on the fused path.  ``doc_start`` (int32 ``[B, T]``) turns on
        intra-document attention masking.

        ``labels`` uses ``-100`` for ignored positions and is already shifted (``labels[:, t]`` is the target of
        position ``t``).  Gradients of ``(ΣCE + z_mult·Σlse²) / loss_divisor`` are accumulated.  Returns the
        device scalars ``ΣCE / loss_divisor`` and ``z_mult·Σlse² / loss_divisor``.

        With peer-memory collectives, the first micro-batch after an optimizer step pulls each unit's foreign shards
        one unit ahead of its use from inside the ``att_proj`` / ``ff_proj`` GEMM launches, and the last micro-batch
        (``is_last``) reduces each unit's gradients from inside the input-gradient GEMMs of the block processed next.
        """
        assert self.fused
        from ..ops import fused_block as fb
        from ..ops import kernels as k
        from ..ops.loss import lm_head_loss

        comm = self.comm
        model, mcfg = self.model, self.model.config
        t = model.transformer
        B, T = input_ids.shape
        M = B * T
        spec = fb.spec_from_config(mcfg)
        cos, sin = fb.rope_tables(T, spec.head_dim, float(mcfg.rope_theta), self.device)
        blocks = model.all_blocks()

        # ---- parameter gather schedule
        gather_queue: List[Unit] = []
        gathered: set = set()
        if comm is not None and self._params_stale:
            gather_queue = self._forward_unit_order()
            self._params_stale = False
        elif comm is None:
            self.gather_params()

        if comm is not None:
            from .peer import BWD_SPANS, FWD_SPANS

        def need(unit: Unit) -> None:
            if unit in gather_queue:  # not prefetched in time: pull it now, in stream order
                gather_queue.remove(unit)
                comm.launch(comm.ag_task(unit))

        def prefetch_kwargs() -> Dict[str, Dict[str, Any]]:
            if not gather_queue:
                return {}
            nxt = gather_queue.pop(0)
            return {name: {"comm": (comm.ag_task(nxt, span=span), comm.comm_ctas)} for name, span in FWD_SPANS.items()}

        if gather_queue:
            need(self._unit_of_module_param(t.wte.weight))
        x = k.embedding_fwd(input_ids, t.wte.weight).view(M, mcfg.d_model)
        saved_list: List[Any] = []
        for i, block in enumerate(blocks):
            if gather_queue:
                need(self._unit_of_module_param(block.att_proj.weight))
            gk = prefetch_kwargs() if gather_queue else None
            w = self._weights_of(block)
            with nvtx_range(f"fwd_block_{i}"):
                if should_checkpoint_block(ac_strategy, i):
                    y, _ = fb.block_forward(spec, w, x, B, T, cos, sin, save=False, gemm_kwargs=gk, doc_start=doc_start)
                    saved_list.append(("ckpt", x))
                else:
                    y, saved = fb.block_forward(spec, w, x, B, T, cos, sin, save=True, gemm_kwargs=gk, doc_start=doc_start,
                                                keep_recomputable=bool(self.keep_recomputable))
                    saved_list.append(("full", saved))
            x = y
        while gather_queue:
            need(gather_queue[0])
        ln_f = t.ln_f
        xn, rstd_f, mean_f = k.norm_fwd(x, ln_f.weight, None, mcfg.layer_norm_eps, spec.rms)
        head = t.wte.weight if mcfg.weight_tying else t.ff_out.weight
        flat_labels = labels.reshape(-1)
        with nvtx_range("lm_head_loss"):
            ce_sum, z_sum, dxn = lm_head_loss(
                xn, head, flat_labels, z_mult=z_mult, grad_scale=1.0 / loss_divisor,
                logit_scale=(1.0 / math.sqrt(mcfg.d_model)) if mcfg.scale_logits else 1.0,
                chunk_rows=int(os.environ.get("OLMO_B200_HEAD_CHUNK", "8192")),
                wgrad=lambda dl, xc: self.matrix_grad(head, dl, xc),
            )
        del xn
        dx = k.norm_bwd(dxn, x, ln_f.weight, rstd_f, mean_f, spec.rms,
                        dweight=None if ln_f.weight is None else self.vector_grad(ln_f.weight))
        del dxn, x

        # ---- gradient reduction schedule (last micro-batch only)
        reduce_now = comm is not None and is_last and not self.reshard
        ready: List[Unit] = []
        final_at: Dict[int, int] = {}
        if reduce_now:
            comm.begin_grad_epoch()
            self._grad_epoch_open = True
            final_at = self._unit_final_points()

            def publish(point: int) -> None:
                for u in self.units:
                    if final_at[u.index] == point:
                        comm.publish_grads(u)
                        u.published = True  # type: ignore[attr-defined]
                        ready.append(u)

            publish(len(blocks))

        def reduce_kwargs() -> Optional[Dict[str, Dict[str, Any]]]:
            if not ready:
                return None
            u = ready.pop(0)
            u.reduced = True  # type: ignore[attr-defined]
            return {name: {"comm": (comm.rs_task(u, span=span), comm.rs_ctas)} for name, span in BWD_SPANS.items()}

        for i in range(len(blocks) - 1, -1, -1):
            kind, payload = saved_list.pop()
            block = blocks[i]
            w = self._weights_of(block)
            if kind == "ckpt":
                # recomputed right before its use: keeping q/k and the activation output costs nothing lasting
                _, payload = fb.block_forward(spec, w, payload, B, T, cos, sin, save=True, doc_start=doc_start, keep_recomputable=True)
            with nvtx_range(f"bwd_block_{i}"):
                dx = fb.block_backward(spec, w, payload, dx, cos, sin, _EngineSink(self, block),
                                       gemm_kwargs=reduce_kwargs() if reduce_now else None)
            del payload
            if reduce_now:
                publish(i)
        k.embedding_bwd(input_ids, dx, self.grad_view(t.wte.weight)[0])
        if reduce_now:
            publish(-1)
            for u in ready:  # whatever found no GEMM to ride on
                u.reduced = True  # type: ignore[attr-defined]
                comm.launch(comm.rs_task(u))
            ready.clear()
        self.note_microbatch_backward()
        if self.keep_recomputable is None and is_last:
            self._decide_keep_recomputable(M, spec, sum(1 for i in range(len(blocks)) if not should_checkpoint_block(ac_strategy, i)))
        return ce_sum / loss_divisor, z_sum * (z_mult / loss_divisor)

    def _decide_keep_recomputable(self, tokens: int, spec, n_blocks: int) -> None:
        """After the first full step the allocator has seen the step's peak, so the memory still free on the device is
        what the extra saved activations may use.  They are kept when they fit with a margin (12 GiB, or a quarter of
        the device if that is smaller)."""
        hidden_half = self.model.config.ff_proj_width // 2
        per_token = (spec.Wq + spec.Wk + (spec.Wk if spec.clip_qkv > 0 else 0) + hidden_half) * 2
        if not spec.norm_after:
            per_token += 2 * self.model.config.d_model * 2
        extra = per_token * tokens * n_blocks
        free, total = torch.cuda.mem_get_info(self.device)
        margin = min(12 << 30, total // 4)
        self.keep_recomputable = free > extra + margin
        log.info(
            "activations that the backward pass can recompute (%.1f GiB per micro-batch) will be %s: %.1f GiB free after the first step",
            extra / 2**30, "kept" if self.keep_recomputable else "recomputed", free / 2**30,
        )

    @torch.no_grad()
    def eval_loss(self, input_ids: torch.Tensor, labels: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Σ CE and the number of scored tokens for one batch, fused path, no gradients."""
        assert self.fused
        from ..ops import fused_block as fb
        from ..ops import kernels as k
        from ..ops.loss import lm_head_loss

        self.gather_params()
        model, mcfg = self.model, self.model.config
        t = model.transformer
        B, T = input_ids.shape
        spec = fb.spec_from_config(mcfg)
        cos, sin = fb.rope_tables(T, spec.head_dim, float(mcfg.rope_theta), self.device)
        x = k.embedding_fwd(input_ids, t.wte.weight).view(B * T, mcfg.d_model)
        for block in model.all_blocks():
            x, _ = fb.block_forward(spec, self._weights_of(block), x, B, T, cos, sin, save=False)
        xn, _, _ = k.norm_fwd(x, t.ln_f.weight, None, mcfg.layer_norm_eps, spec.rms, save_stats=False)
        head = t.wte.weight if mcfg.weight_tying else t.ff_out.weight
        ce_sum, _, _ = lm_head_loss(xn, head, labels.reshape(-1), need_grad=False,
                                    logit_scale=(1.0 / math.sqrt(mcfg.d_model)) if mcfg.scale_logits else 1.0)
        return ce_sum, (labels != -100).sum()

    # ------------------------------------------------------------------------ state dicts
    def full_tensor(self, unit: Unit, shard: torch.Tensor) -> torch.Tensor:
        """Gather an fp32 per-shard tensor of ``unit`` to its full (padded) length on every rank."""
        if not self.is_sharded:
            return shard
        out = torch.empty(unit.numel, dtype=shard.dtype, device=shard.device)
        if self.device.type == "cuda":
            dist.all_gather_into_tensor(out, shard.contiguous(), group=self.shard_group)
        else:
            chunks = [torch.empty_like(shard) for _ in range(self.shard_world)]
            dist.all_gather(chunks, shard.contiguous(), group=self.shard_group)
            torch.cat(chunks, out=out)
        return out

    def full_model_state_dict(self, rank0_only: bool = True, cpu: bool = True) -> Dict[str, torch.Tensor]:
        """``{FQN: fp32 tensor}`` of the whole model, assembled from the master shards."""
        out: Dict[str, torch.Tensor] = {}
        keep = (not rank0_only) or self.rank == 0
        for unit in self.units:
            flat = self.full_tensor(unit, unit.master)
            if keep:
                for s in unit.slots:
                    tsr = flat[s.offset : s.offset + s.numel].view(s.shape)
                    out[s.name] = tsr.cpu().clone() if cpu else tsr.clone()
            del flat
        if self.model.config.weight_tying and keep and "transformer.wte.weight" in out:
            pass  # tied head has no separate entry, like nn.Module.state_dict() of the reference
        return out

    def load_full_model_state_dict(self, state: Dict[str, torch.Tensor]) -> None:
        """Scatter full tensors into the master shards (every rank passes the same dict) and refresh all copies."""
        missing = [s.name for u in self.units for s in u.slots if s.name not in state]
        unexpected = [kname for kname in state if kname not in self._unit_of_param]
        if missing or unexpected:
            raise KeyError(f"state dict mismatch: missing {missing[:5]}, unexpected {unexpected[:5]}")
        for unit in self.units:
            lo = self.shard_rank * unit.shard_size
            hi = lo + unit.shard_size
            for s in unit.slots:
                src = state[s.name].reshape(-1)
                a, b = max(s.offset, lo), min(s.offset + s.numel, hi)
                if b > a:
                    unit.master[a - lo : b - lo].copy_(src[a - s.offset : b - s.offset].to(unit.master.device, torch.float32))
                unit.full[s.offset : s.offset + s.numel].copy_(src.to(unit.full.device, unit.full.dtype))
        self._params_stale = False

    def param_shard_ranges(self) -> Dict[str, Tuple[int, int, int]]:
        """``FQN -> (start, end, numel)``: the element range of the parameter held by this rank."""
        out = {}
        for unit in self.units:
            lo = self.shard_rank * unit.shard_size
            hi = lo + unit.shard_size
            for s in unit.slots:
                a, b = max(s.offset, lo), min(s.offset + s.numel, hi)
                out[s.name] = (max(a - s.offset, 0), max(b - s.offset, 0) if b > a else max(a - s.offset, 0), s.numel)
        return out


class _EngineSink:
    """Gradient sink of the fused backward pass: points each block parameter at its slice of the engine's buffers."""

    def __init__(self, engine: FlatShardEngine, block: OLMoBlock):
        self.engine = engine
        self.params = {
            "att_proj": block.att_proj.weight, "attn_out": block.attn_out.weight, "ff_proj": block.ff_proj.weight,
            "ff_out": block.ff_out.weight, "attn_norm": block.attn_norm.weight, "ff_norm": block.ff_norm.weight,
            "q_norm": None if block.q_norm is None else block.q_norm.weight,
            "k_norm": None if block.k_norm is None else block.k_norm.weight,
        }

    def matrix(self, name: str, dy: torch.Tensor, x: torch.Tensor) -> None:
        self.engine.matrix_grad(self.params[name], dy, x)

    def vector(self, name: str, like: torch.Tensor) -> torch.Tensor:
        return self.engine.vector_grad(self.params[name])


class ShardedModel(nn.Module):
    """``nn.Module`` façade over the engine: what the trainer holds as ``dist_model``."""

    def __init__(self, engine: FlatShardEngine):
        super().__init__()
        self.engine = engine
        self.module = engine.model

    @property
    def is_flat_sharded(self) -> bool:
        return self.engine.is_sharded

    @property
    def process_group(self):
        return self.engine.process_group

    def named_parameters_for_optimizer(self):
        return self.engine.named_parameters_for_optimizer()

    def forward(self, *args, **kwargs) -> OLMoOutput:
        self.engine.gather_params()
        return self.module(*args, **kwargs)


def build_sharded_model(model: OLMo, cfg: TrainConfig, device: torch.device, **kwargs) -> ShardedModel:
    return ShardedModel(FlatShardEngine(model, cfg, device, **kwargs))
