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
shard inside a replica group and all-reduce across groups, ``NO_SHARD`` and ``ddp`` replicate.

Schedules (fused path with peer-memory collectives)
---------------------------------------------------
``resident``  the gathered compute copy and the full-size fp32 gradient accumulator of *every* unit stay allocated
              (6 bytes per parameter that do not shrink with the number of ranks).  Gradients of all micro-batches are
              accumulated locally, so an optimizer step pays one gather and one reduce-scatter per unit.  This is what
              ``SHARD_GRAD_OP`` asks for, and what ``FULL_SHARD`` gets while it fits, because it is the faster schedule.
``sharded``   the ``FULL_SHARD`` schedule proper (reference: ``scripts/train.py:210-220``, and ``olmo/train.py:796-803``:
              no ``no_sync`` on the FSDP path, i.e. a reduction per micro-batch).  Units that consist of transformer
              blocks are *streamed*: a rank keeps only its shards of them, two full-size parameter slots and three
              full-size gradient slots.  Every micro-batch gathers block *i+1* from inside block *i*'s four forward GEMMs,
              gathers block *i-1* again from inside block *i*'s weight-gradient GEMMs in the backward pass, and
              reduce-scatters block *i*'s gradients from inside block *i-1*'s input-gradient GEMMs into the fp32 gradient
              shard (summing Σg² on the last micro-batch).  The embedding, the final norm and the output projection are
              used at the two ends of the pass, where there is no GEMM to hide their traffic behind; they stay resident
              and are gathered / reduced once per step.

``OLMO_B200_SCHEDULE=resident|sharded|auto`` selects it (``auto``, the default: ``sharded`` for ``FULL_SHARD`` when the
resident set would take more than 60 % of the device together with the optimizer shards).
"""
from __future__ import annotations

import logging
import math
import os
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any, Dict, Iterator, List, Optional, Tuple

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
from ..torch_util import get_global_rank, get_world_size, nvtx_range

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
    streamed: bool = False  # sharded schedule: no resident `full` / `gfull`; gathered into rotating slots
    stream_pos: int = -1  # position among the streamed units in forward order
    zero_ranges: List[Tuple[int, int]] = field(default_factory=list, repr=False)  # what is not a matrix: vectors, padding

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
        sched = os.environ.get("OLMO_B200_SCHEDULE", "auto").strip().lower()
        if os.environ.get("OLMO_B200_RESHARD", "0") not in ("0", "", "false"):
            sched = "sharded"  # older spelling of OLMO_B200_SCHEDULE=sharded, still honoured
        if sched not in ("auto", "resident", "sharded"):
            raise OLMoConfigurationError("OLMO_B200_SCHEDULE must be one of auto, resident, sharded")
        self._schedule_request = sched
        self.schedule = "resident"  # decided in _build, once the unit sizes are known
        self.stream: Optional["_StreamState"] = None
        self.phase_timer: Any = None  # optional object with ``mark(name)``: CUDA events at phase boundaries (bench.py)
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
    def _collect_units(self) -> List[Tuple[str, List[Tuple[str, nn.Parameter, nn.Module, str]], List[nn.Module]]]:
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
                out.append((uname, entries, list(modules)))
        return out

    def _decide_schedule(self, use_peer: bool) -> str:
        if not use_peer or not self.is_sharded:
            return "resident"
        if self.num_replicas > 1:
            if self._schedule_request == "sharded":
                log.warning("the sharded schedule covers one shard group spanning the job; with model replicas the resident schedule is used")
            return "resident"
        req = self._schedule_request
        if req == "auto":
            if self.sharding_strategy != ShardingStrategy.FULL_SHARD:
                return "resident"
            P = sum(u.numel for u in self.units)
            need = 6 * P + 16 * P // self.shard_world
            req = "sharded" if need > 0.6 * torch.cuda.get_device_properties(self.device).total_memory else "resident"
        return req

    def _materialise_unit(self, uname: str, entries, seed: int) -> None:
        """Allocate and initialise the parameters of one unit in fp32 on the device.  Every module's random stream is a
        function of ``(seed, module name)`` only, so the weights do not depend on the world size, the sharding strategy
        or the wrapping, and no rank ever holds more than its shards plus one unit."""
        dev = self.device
        mine = {(id(owner), attr) for _, _, owner, attr in entries}
        for name, p, owner, attr in entries:
            if p.is_meta:
                owner._parameters[attr] = nn.Parameter(torch.empty(p.shape, dtype=torch.float32, device=dev), requires_grad=p.requires_grad)
        def all_mine(m: nn.Module) -> bool:
            return all((id(sub), attr) in mine for sub in m.modules() for attr, _ in sub.named_parameters(recurse=False))

        self.model.reset_parameters(only={id(m) for m in self.model.initialisable_modules() if all_mine(m)}, seed=seed)

    def _build(self, seed: int) -> None:
        model, dev = self.model, self.device
        # 1. flat layout (shapes only: parameters may still be on the meta device)
        meta = any(p.is_meta for p in model.parameters())
        if not meta:
            model.to(dev)
        sw = self.shard_world
        collected = self._collect_units()
        for index, (uname, entries, _mods) in enumerate(collected):
            offset = 0
            slots = []
            for name, p, owner, attr in entries:
                slots.append(ParamSlot(name, p.shape, p.numel(), offset, owner, attr))
                offset = _round_up(offset + p.numel(), ALIGN)
            total = _round_up(max(offset, 1), sw * 1024)
            unit = Unit(uname, index, slots, total, total // sw)
            self.units.append(unit)
        # 2. schedule; which units are streamed
        use_peer = (
            self.world > 1 and dev.type == "cuda" and self.fused
            and os.environ.get("OLMO_B200_FUSED_COMM", "1").strip().lower() not in ("0", "false", "no", "off")
        )
        self.schedule = self._decide_schedule(use_peer)
        if self.schedule == "sharded":
            block_prefixes = ("transformer.blocks.", "transformer.block_groups.")
            pos = 0
            for unit in self.units:
                if unit.slots and all(s.name.startswith(block_prefixes) for s in unit.slots):
                    unit.streamed, unit.stream_pos = True, pos
                    pos += 1
                    cur, gaps = 0, []
                    for sl in unit.slots:  # everything that is not a matrix is cleared before each backward use
                        if len(sl.shape) >= 2:
                            if sl.offset > cur:
                                gaps.append((cur, sl.offset))
                            cur = sl.offset + sl.numel
                    if cur < unit.numel:
                        gaps.append((cur, unit.numel))
                    unit.zero_ranges = gaps
            if pos == 0:
                self.schedule = "resident"
        # 3. buffers; module parameters become views of `full` (placeholders on the meta device for streamed units)
        if use_peer:
            from .peer import PeerComm

            self.comm = PeerComm.create(self)
        for unit, (uname, entries, _mods) in zip(self.units, collected):
            if meta:
                self._materialise_unit(uname, entries, seed)
            S, P = unit.shard_size, unit.numel
            lo = self.shard_rank * S
            flat = torch.zeros(P, dtype=torch.float32, device=dev)
            for sl in unit.slots:
                flat[sl.offset : sl.offset + sl.numel].copy_(getattr(sl.owner, sl.attr).detach().reshape(-1).float())
            unit.master = flat[lo : lo + S].clone() if sw > 1 else flat
            unit.grad = torch.zeros(S, dtype=torch.float32, device=dev)
            streamed = unit.streamed and self.comm is not None
            unit.streamed = streamed
            if streamed:
                unit.full = unit.gfull = None  # type: ignore[assignment]
                unit.lowp = self.comm.lowp_view(unit)
                unit.lowp.copy_(unit.master)
            elif self.comm is not None:
                unit.full = self.comm.full_view(unit.index, P)
                unit.full.copy_(flat)
                unit.gfull = self.comm.gfull_view(unit.index, P)
            else:
                unit.full = flat.to(self.compute_dtype) if (self.compute_dtype != torch.float32 or sw > 1) else flat.clone()
                unit.gfull = unit.grad if sw == 1 else None  # type: ignore[assignment]
            if not streamed:
                unit.lowp = unit.full[lo : lo + S] if sw > 1 else unit.full
            for sl in unit.slots:
                if streamed:
                    view = torch.empty(sl.shape, dtype=self.compute_dtype, device="meta")
                else:
                    view = unit.full[sl.offset : sl.offset + sl.numel].view(sl.shape)
                param = nn.Parameter(view, requires_grad=not self.fused)
                param._ob_unit = unit  # type: ignore[attr-defined]
                param._ob_slot = sl  # type: ignore[attr-defined]
                sl.owner._parameters[sl.attr] = param
                self._unit_of_param[sl.name] = (unit, sl)
            del flat
        if self.comm is None or not any(u.streamed for u in self.units):
            self.schedule = "resident"
        if dev.type == "cuda":
            torch.cuda.empty_cache()
        # 4. optimizer-facing parameters: one per (parameter ∩ local shard)
        for unit in self.units:
            lo = self.shard_rank * unit.shard_size
            hi = lo + unit.shard_size
            for sl in unit.slots:
                a, b = max(sl.offset, lo), min(sl.offset + sl.numel, hi)
                if b > a:
                    data = unit.master[a - lo : b - lo]
                    gview = unit.grad[a - lo : b - lo]
                    if b - a == sl.numel:
                        data, gview = data.view(sl.shape), gview.view(sl.shape)
                else:
                    data = unit.master[0:0]
                    gview = unit.grad[0:0]
                p = nn.Parameter(data, requires_grad=True)
                p.grad = gview
                p._ob_range = (unit.index, a - lo, max(b, a) - lo)  # type: ignore[attr-defined]
                self._opt_params.append((sl.name, p))
        self._params_stale = False  # `full` was filled from the initial weights
        if self.fused:
            self._setup_fused()
        if self.is_sharded and self.comm is None:
            for unit in self.units:
                unit.gfull = torch.zeros(unit.numel, dtype=torch.float32, device=dev)
        if meta:
            torch.manual_seed(seed)
            if dev.type == "cuda":
                torch.cuda.manual_seed(seed)
        if self.schedule == "sharded":
            self.stream = _StreamState(self)
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.shard_group)  # every rank's shards are in place before anyone gathers
        log.info(
            "FlatShardEngine: %d units, %.2fB parameters, shard world %d, replicas %d, %s path, %s schedule",
            len(self.units), sum(s.numel for u in self.units for s in u.slots) / 1e9, self.shard_world, self.num_replicas,
            "fused" if self.fused else "portable", self.schedule,
        )

    # ----------------------------------------------------------------------- optimizer side
    def _mark(self, name: str) -> None:
        if self.phase_timer is not None:
            self.phase_timer.mark(name)

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

        self._mark("grad_sync")
        self.finish_grad_sync()
        comm = self.comm
        if comm is not None and comm.fuse_sumsq:
            # every shard received its last addition of the step from a reduce-scatter kernel that also summed its squares
            torch.sum(comm.rs_partials, dim=0, keepdim=True, out=self._sumsq)
        else:
            for i, unit in enumerate(self.units):
                k.sumsq(unit.grad, self._sumsq, accumulate=i > 0)
        self._mark("barrier_wait")
        if self.comm is not None:  # also the end-of-step barrier of the whole job, so it runs even when nothing is sharded
            self.comm.all_reduce_scalar_(self._sumsq)
        elif self.is_sharded:
            dist.all_reduce(self._sumsq, group=process_group or self.shard_group)
        self._mark("clip")
        k.clip_coef(self._sumsq, float(max_norm) if max_norm is not None else float("inf"), self.clip_coef, self._norm_out)
        return self._norm_out[0].clone()

    def fused_optimizer_step(self, optim, kind: str, gscale: Optional[torch.Tensor]) -> None:
        from ..ops import kernels as k

        self._mark("optimizer")
        self.finish_grad_sync()
        self._ensure_fused_state(optim, kind)
        self._refresh_segments(optim)
        # one step count for the whole model: per-parameter counters can lag on ranks whose shard of a parameter is empty
        # (the per-parameter optimizer skips those), and every rank must apply the same bias correction
        step = 1 + max((int(optim.state[p]["step"].item()) for _, p in self._opt_params), default=0)
        for _, p in self._opt_params:
            optim.state[p]["step"].fill_(float(step))
        groups = optim.param_groups
        if any(g["betas"] != groups[0]["betas"] or g.get("eps", 0.0) != groups[0].get("eps", 0.0) for g in groups[1:]):
            raise OLMoConfigurationError("the fused optimizer kernels take one (betas, eps) for all parameter groups")
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
        self._mark("end")

    def verify_collectives_against_nccl(self) -> Dict[str, Any]:
        """Check the peer-memory collectives of the step that just ran against NCCL on the same local buffers.

        Call between an optimizer step and the next ``zero_grad``.  Resident units: the fp32 gradient shard must equal
        ``reduce_scatter(gfull) / world`` (``gfull`` still holds this rank's unreduced gradients of the step), and after
        a gather ``full`` must equal ``all_gather(lowp)`` bit for bit.  Streamed units: a gather into a parameter slot is
        compared with NCCL's; their gradient slots have been reused by then, so their reduction is covered by the
        multi-GPU tests instead.  Only local memory is handed to NCCL.  Collective: every rank calls it."""
        assert self.comm is not None
        world = self.shard_world
        worst_rs, bad_ag, checked_rs, checked_ag = 0.0, 0, 0, 0
        self.gather_params()
        for unit in self.units:
            shard = unit.lowp.contiguous()
            ref = torch.empty(unit.numel, dtype=shard.dtype, device=self.device)
            if world > 1:
                dist.all_gather_into_tensor(ref, shard, group=self.shard_group)
            else:
                ref.copy_(shard)
            if unit.streamed:
                st = self.stream
                st.content[unit.stream_pos % st.n_full] = None
                st.ensure(unit.stream_pos)
                mine = self.comm.full_slot(unit.stream_pos % st.n_full)[: unit.numel]
            else:
                mine = unit.full
            bad_ag += int((mine.view(torch.int16) != ref.view(torch.int16)).sum().item()) if shard.dtype == torch.bfloat16 else int((mine != ref).sum().item())
            checked_ag += unit.numel
            del ref
            if not unit.streamed and getattr(unit, "reduced", False):
                if world > 1:
                    out = torch.empty(unit.shard_size, dtype=torch.float32, device=self.device)
                    dist.reduce_scatter_tensor(out, unit.gfull.clone(), group=self.shard_group)
                else:
                    out = unit.gfull.clone()
                if self.num_replicas > 1:
                    dist.all_reduce(out, group=self.replica_group)
                out.div_(self.world)
                denom = out.abs().max().clamp_min(1e-30)
                worst_rs = max(worst_rs, float(((unit.grad - out).abs().max() / denom).item()))
                checked_rs += unit.shard_size
        t = torch.tensor([worst_rs, float(bad_ag)], device=self.device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        worst_rs, bad_ag = float(t[0]), int(t[1])
        return {
            "ok": bool(worst_rs < 1e-5 and bad_ag == 0), "reduce_scatter_max_rel_err_vs_nccl": worst_rs,
            "all_gather_mismatched_elements_vs_nccl": bad_ag, "gradient_elements_checked": checked_rs,
            "parameter_elements_checked": checked_ag, "schedule": self.schedule,
        }

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
                unit.gfull.zero_()  # streamed units have none: their gradient slots are overwritten, not accumulated into
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
                self.comm.all_gather_units([u for u in self.units if not u.streamed])
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
            pending = [u for u in self.units if not u.streamed and not getattr(u, "reduced", False)]
            if pending:
                if not self._grad_epoch_open:
                    self.comm.begin_grad_epoch()
                for u in pending:
                    if not getattr(u, "published", False):
                        self.comm.publish_grads(u)
                self.comm.reduce_scatter_units(pending, scale=1.0 / world)
                for u in pending:
                    self.comm.finish_replicas(u)
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
        if self.stream is not None:
            return self._train_microbatch_streamed(input_ids, labels, loss_divisor, z_mult, ac_strategy, is_last, doc_start)
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
            if self.is_sharded:
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
        self._mark("forward")
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
        self._mark("backward")
        dx = k.norm_bwd(dxn, x, ln_f.weight, rstd_f, mean_f, spec.rms,
                        dweight=None if ln_f.weight is None else self.vector_grad(ln_f.weight))
        del dxn, x

        # ---- gradient reduction schedule (last micro-batch only)
        reduce_now = comm is not None and is_last
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

        riding: List[Unit] = []

        def reduce_kwargs() -> Optional[Dict[str, Dict[str, Any]]]:
            if not ready:
                return None
            u = ready.pop(0)
            u.reduced = True  # type: ignore[attr-defined]
            riding.append(u)
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
                while riding:  # the block's GEMMs carried this unit's reduce-scatter: now the replica group's turn
                    comm.finish_replicas(riding.pop())
                publish(i)
        k.embedding_bwd(input_ids, dx, self.grad_view(t.wte.weight)[0])
        if reduce_now:
            publish(-1)
            for u in ready:  # whatever found no GEMM to ride on
                u.reduced = True  # type: ignore[attr-defined]
                comm.launch(comm.rs_task(u))
                comm.finish_replicas(u)
            ready.clear()
        self.note_microbatch_backward()
        if self.keep_recomputable is None and is_last:
            self._decide_keep_recomputable(M, spec, sum(1 for i in range(len(blocks)) if not should_checkpoint_block(ac_strategy, i)))
        return ce_sum / loss_divisor, z_sum * (z_mult / loss_divisor)

    def _train_microbatch_streamed(self, input_ids, labels, loss_divisor, z_mult, ac_strategy, is_last, doc_start):
        """One micro-batch of the sharded schedule: block units pass through the parameter and gradient slots, their
        collectives ride on the block GEMMs of every micro-batch (see the module docstring)."""
        from ..ops import fused_block as fb
        from ..ops import kernels as k
        from ..ops.loss import lm_head_loss
        from .peer import BWD_SPANS, FWD_SPANS, WGRAD_SPANS

        comm, st = self.comm, self.stream
        model, mcfg = self.model, self.model.config
        t = model.transformer
        B, T = input_ids.shape
        M = B * T
        spec = fb.spec_from_config(mcfg)
        cos, sin = fb.rope_tables(T, spec.head_dim, float(mcfg.rope_theta), self.device)
        blocks = model.all_blocks()
        n_stream = len(st.seq)

        if self._params_stale:  # resident units (embedding, final norm, head): once per optimizer step
            comm.all_gather_units([u for u in self.units if not u.streamed])
            self._params_stale = False

        # ---- forward
        self._mark("forward")
        x = k.embedding_fwd(input_ids, t.wte.weight).view(M, mcfg.d_model)
        saved_list: List[Any] = []
        for i, block in enumerate(blocks):
            pos = st.block_pos[i]
            gk = None
            if pos >= 0:
                st.ensure(pos)
                if st.last_block[pos] == i and pos + 1 < n_stream:
                    gk = st.prefetch(pos + 1, FWD_SPANS)
            w = st.weights(i) if pos >= 0 else self._weights_of(block)
            with nvtx_range(f"fwd_block_{i}"):
                if should_checkpoint_block(ac_strategy, i):
                    y, _ = fb.block_forward(spec, w, x, B, T, cos, sin, save=False, gemm_kwargs=gk, doc_start=doc_start)
                    saved_list.append(("ckpt", x))
                else:
                    y, saved = fb.block_forward(spec, w, x, B, T, cos, sin, save=True, gemm_kwargs=gk, doc_start=doc_start,
                                                keep_recomputable=bool(self.keep_recomputable))
                    saved_list.append(("full", saved))
            x = y
        ln_f = t.ln_f
        xn, rstd_f, mean_f = k.norm_fwd(x, ln_f.weight, None, mcfg.layer_norm_eps, spec.rms)
        head = t.wte.weight if mcfg.weight_tying else t.ff_out.weight
        with nvtx_range("lm_head_loss"):
            ce_sum, z_sum, dxn = lm_head_loss(
                xn, head, labels.reshape(-1), z_mult=z_mult, grad_scale=1.0 / loss_divisor,
                logit_scale=(1.0 / math.sqrt(mcfg.d_model)) if mcfg.scale_logits else 1.0,
                chunk_rows=int(os.environ.get("OLMO_B200_HEAD_CHUNK", "8192")),
                wgrad=lambda dl, xc: self.matrix_grad(head, dl, xc),
            )
        del xn
        self._mark("backward")
        dx = k.norm_bwd(dxn, x, ln_f.weight, rstd_f, mean_f, spec.rms,
                        dweight=None if ln_f.weight is None else self.vector_grad(ln_f.weight))
        del dxn, x

        # ---- resident units are reduced once per step, by stand-alone launches on the last micro-batch
        final_at: Dict[int, int] = {}
        if is_last:
            comm.begin_grad_epoch()
            final_at = {u: p for u, p in self._unit_final_points().items() if not self.units[u].streamed}

        def reduce_resident(point: int) -> None:
            for u in self.units:
                if final_at.get(u.index) == point:
                    comm.publish_grads(u)
                    comm.launch(comm.rs_task(u))
                    u.reduced = True  # type: ignore[attr-defined]

        if is_last:
            reduce_resident(len(blocks))

        # ---- backward
        for i in range(len(blocks) - 1, -1, -1):
            kind, payload = saved_list.pop()
            block = blocks[i]
            pos = st.block_pos[i]
            if pos < 0:  # a block that lives in a resident unit
                w = self._weights_of(block)
                if kind == "ckpt":
                    _, payload = fb.block_forward(spec, w, payload, B, T, cos, sin, save=True, doc_start=doc_start, keep_recomputable=True)
                with nvtx_range(f"bwd_block_{i}"):
                    dx = fb.block_backward(spec, w, payload, dx, cos, sin, _EngineSink(self, block), gemm_kwargs=st.rs_kwargs(BWD_SPANS, is_last))
                st.rs_done()
                del payload
                if is_last:
                    reduce_resident(i)
                continue
            st.ensure(pos)
            w = st.weights(i)
            if kind == "ckpt":
                _, payload = fb.block_forward(spec, w, payload, B, T, cos, sin, save=True, doc_start=doc_start, keep_recomputable=True)
            if st.last_block[pos] == i:  # first block of this unit in backward order: take a gradient slot
                st.open_grads(pos)
            wk = None
            if st.first_block[pos] == i and pos - 1 >= 0:  # re-gather the unit the backward pass needs next
                wk = st.prefetch(pos - 1, WGRAD_SPANS)
            with nvtx_range(f"bwd_block_{i}"):
                dx = fb.block_backward(spec, w, payload, dx, cos, sin, st.sink(i, wk),
                                       gemm_kwargs=st.rs_kwargs(BWD_SPANS, is_last))
            st.rs_done()
            del payload
            if st.first_block[pos] == i:  # the unit's gradients of this micro-batch are complete
                st.publish_grads(pos, is_last)
        k.embedding_bwd(input_ids, dx, self.grad_view(t.wte.weight)[0])
        st.flush_rs(is_last)
        if is_last:
            reduce_resident(-1)
            for u in self.units:
                if not u.streamed and not getattr(u, "reduced", False):
                    comm.publish_grads(u)
                    comm.launch(comm.rs_task(u))
                    u.reduced = True  # type: ignore[attr-defined]
        self._grads_pending = False
        self._microbatches_since_reduce += 1
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
        st = self.stream
        for i, block in enumerate(model.all_blocks()):
            gk = None
            if st is not None and st.block_pos[i] >= 0:
                from .peer import FWD_SPANS

                pos = st.block_pos[i]
                st.ensure(pos)
                if st.last_block[pos] == i and pos + 1 < len(st.seq):
                    gk = st.prefetch(pos + 1, FWD_SPANS)
                w = st.weights(i)
            else:
                w = self._weights_of(block)
            x, _ = fb.block_forward(spec, w, x, B, T, cos, sin, save=False, gemm_kwargs=gk)
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
                if unit.full is not None:
                    unit.full[s.offset : s.offset + s.numel].copy_(src.to(unit.full.device, unit.full.dtype))
            if unit.streamed:
                unit.lowp.copy_(unit.master)
        self._params_stale = False
        self.params_changed(resident_current=True)

    def params_changed(self, resident_current: bool = False) -> None:
        """The master shards were overwritten from outside the optimizer (checkpoint restore, state-dict load): refresh
        what peers gather from and, with peer-memory collectives, open a new parameter epoch once every rank is done."""
        if not resident_current:
            for unit in self.units:
                if unit.lowp.data_ptr() != unit.master.data_ptr():
                    unit.lowp.copy_(unit.master)
            self._params_stale = True
        if self.comm is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.shard_group)
            self.comm.publish_params()

    @contextmanager
    def summon_full_params(self) -> Iterator[None]:
        """Inside the context the module parameters of streamed units are real, gathered tensors (compute dtype), so the
        plain ``nn.Module`` forward (generation, module-level evaluation, tracing) works.  A no-op in the resident
        schedule.  Collective: every rank of the shard group must enter."""
        streamed = [u for u in self.units if u.streamed]
        if not streamed:
            yield
            return
        held = []
        for unit in streamed:
            full = torch.empty(unit.numel, dtype=unit.lowp.dtype, device=self.device)
            dist.all_gather_into_tensor(full, unit.lowp.contiguous(), group=self.shard_group)
            for sl in unit.slots:
                placeholder = sl.owner._parameters[sl.attr]
                real = nn.Parameter(full[sl.offset : sl.offset + sl.numel].view(sl.shape), requires_grad=False)
                real._ob_unit, real._ob_slot = unit, sl  # type: ignore[attr-defined]
                sl.owner._parameters[sl.attr] = real
                held.append((sl, placeholder))
        try:
            yield
        finally:
            for sl, placeholder in held:
                sl.owner._parameters[sl.attr] = placeholder

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


class _StreamState:
    """Book-keeping of the sharded schedule: which streamed unit sits in which parameter slot, which gradient slot a
    unit writes to, and the reduce-scatter that is waiting for GEMMs to ride on."""

    def __init__(self, engine: FlatShardEngine):
        from .peer import N_FULL_SLOTS, N_GSLOTS

        self.engine = engine
        self.comm = engine.comm
        self.n_full, self.n_g = N_FULL_SLOTS, N_GSLOTS
        self.seq: List[Unit] = sorted((u for u in engine.units if u.streamed), key=lambda u: u.stream_pos)
        self.content: List[Optional[Tuple[int, int]]] = [None] * self.n_full  # (stream position, parameter epoch)
        self.block_pos: List[int] = []
        self.block_slots: List[Dict[str, ParamSlot]] = []
        self.first_block: Dict[int, int] = {}
        self.last_block: Dict[int, int] = {}
        for i, block in enumerate(engine.model.all_blocks()):
            params = {
                "att_proj": block.att_proj.weight, "attn_out": block.attn_out.weight, "ff_proj": block.ff_proj.weight,
                "ff_out": block.ff_out.weight, "attn_norm": block.attn_norm.weight, "ff_norm": block.ff_norm.weight,
                "q_norm": None if block.q_norm is None else block.q_norm.weight,
                "k_norm": None if block.k_norm is None else block.k_norm.weight,
            }
            unit: Unit = params["att_proj"]._ob_unit  # type: ignore[union-attr]
            pos = unit.stream_pos if unit.streamed else -1
            self.block_pos.append(pos)
            self.block_slots.append({key: p._ob_slot for key, p in params.items() if p is not None})  # type: ignore[attr-defined]
            if pos >= 0:
                self.first_block.setdefault(pos, i)
                self.last_block[pos] = i
        self._weights: Dict[Tuple[int, int], Dict[str, Optional[torch.Tensor]]] = {}
        self.gslot_of: Dict[int, int] = {}  # stream position -> gradient slot of the current micro-batch
        self.pending: Optional[Unit] = None  # unit whose gradients are published but not yet reduced
        self._riding: Optional[Unit] = None

    # ---- parameters
    def present(self, pos: int) -> bool:
        return self.content[pos % self.n_full] == (pos, self.comm.param_epoch)

    def ensure(self, pos: int) -> None:
        """Gather unit ``pos`` with a stand-alone launch unless its slot already holds the current weights."""
        if not self.present(pos):
            self.comm.launch(self.comm.stream_ag_task(self.seq[pos], pos % self.n_full))
            self.content[pos % self.n_full] = (pos, self.comm.param_epoch)

    def prefetch(self, pos: int, spans: Dict[str, Tuple[int, int, int]]) -> Optional[Dict[str, Dict[str, Any]]]:
        """GEMM keyword arguments that make the named GEMMs carry the gather of unit ``pos`` (``None`` if it is there)."""
        if self.present(pos):
            return None
        slot = pos % self.n_full
        self.content[slot] = (pos, self.comm.param_epoch)
        unit = self.seq[pos]
        return {name: {"comm": (self.comm.stream_ag_task(unit, slot, span=span), self.comm.comm_ctas)} for name, span in spans.items()}

    def weights(self, block_index: int) -> Dict[str, Optional[torch.Tensor]]:
        pos = self.block_pos[block_index]
        slot = pos % self.n_full
        hit = self._weights.get((block_index, slot))
        if hit is None:
            buf = self.comm.full_slot(slot)
            hit = {key: None for key in ("att_proj", "attn_out", "ff_proj", "ff_out", "attn_norm", "ff_norm", "q_norm", "k_norm")}
            for key, sl in self.block_slots[block_index].items():
                hit[key] = buf[sl.offset : sl.offset + sl.numel].view(sl.shape)
            self._weights[(block_index, slot)] = hit
        return hit

    # ---- gradients
    def open_grads(self, pos: int) -> None:
        """Take the next gradient slot for unit ``pos``: wait until peers have drained its previous use, then clear the
        parts that kernels add into (norm weights, padding); matrices are written with plain stores."""
        g = pos % self.n_g
        self.comm.open_gslot(g)
        self.gslot_of[pos] = g
        buf = self.comm.gslot(g)
        for a, b in self.seq[pos].zero_ranges:
            buf[a:b].zero_()

    def sink(self, block_index: int, wgrad_comm: Optional[Dict[str, Dict[str, Any]]]) -> "_StreamSink":
        pos = self.block_pos[block_index]
        return _StreamSink(self.comm.gslot(self.gslot_of[pos]), self.block_slots[block_index], wgrad_comm or {})

    def publish_grads(self, pos: int, is_last: bool) -> None:
        if self.pending is not None:  # nothing carried the previous unit's reduction: do it now
            self.flush_rs(is_last)
        self.comm.publish_gslot(self.gslot_of[pos])
        self.pending = self.seq[pos]

    def rs_kwargs(self, spans: Dict[str, Tuple[int, int, int]], is_last: bool) -> Optional[Dict[str, Dict[str, Any]]]:
        """GEMM keyword arguments that make the input-gradient GEMMs of the next block carry the pending reduction."""
        if self.pending is None:
            return None
        unit, self.pending = self.pending, None
        self._riding = unit
        g = self.gslot_of[unit.stream_pos]
        return {name: {"comm": (self.comm.stream_rs_task(unit, g, span=span, with_sumsq=is_last), self.comm.rs_ctas)} for name, span in spans.items()}

    def rs_done(self) -> None:
        """Call after the block whose GEMMs carried a reduction: tell peers this rank has finished reading the slot."""
        if self._riding is not None:
            self.comm.release_gslot(self.gslot_of[self._riding.stream_pos])
            self._riding = None

    def flush_rs(self, is_last: bool) -> None:
        """Stand-alone reduction of the unit that found no GEMM to ride on (the first block's unit)."""
        if self.pending is not None:
            unit, self.pending = self.pending, None
            g = self.gslot_of[unit.stream_pos]
            self.comm.launch(self.comm.stream_rs_task(unit, g, with_sumsq=is_last))
            self.comm.release_gslot(g)


class _StreamSink:
    """Gradient sink of a streamed block: matrices are stored (not accumulated) into the unit's gradient slot, and the
    weight-gradient GEMMs may carry the re-gather of the next unit."""

    def __init__(self, gbuf: torch.Tensor, slots: Dict[str, ParamSlot], comm_kwargs: Dict[str, Dict[str, Any]]):
        self.gbuf, self.slots, self.comm_kwargs = gbuf, slots, comm_kwargs

    def _view(self, name: str) -> torch.Tensor:
        sl = self.slots[name]
        return self.gbuf[sl.offset : sl.offset + sl.numel].view(sl.shape)

    def matrix(self, name: str, dy: torch.Tensor, x: torch.Tensor) -> None:
        from ..ops import kernels as k

        k.gemm(dy, x, a_trans=True, b_trans=True, epilogue=k.EPI_F32_STORE, out=self._view(name), **self.comm_kwargs.get(name, {}))

    def vector(self, name: str, like: torch.Tensor) -> torch.Tensor:
        return self._view(name)


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
        with self.engine.summon_full_params():
            return self.module(*args, **kwargs)


def build_sharded_model(model: OLMo, cfg: TrainConfig, device: torch.device, **kwargs) -> ShardedModel:
    return ShardedModel(FlatShardEngine(model, cfg, device, **kwargs))
