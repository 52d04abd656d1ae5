"""
Peer-memory runtime of the flat-shard engine: symmetric buffers, flags, and the CommTask descriptors consumed by the
kernels in ``csrc/comm.cuh``.

Every rank allocates, in CUDA symmetric memory (``torch.distributed._symmetric_memory``: VMM allocations whose handles
are exchanged once over the process group's store and mapped into every peer),

* ``full_all``   the compute-dtype copy of every unit, end to end.  A rank's own shard of a unit lives *inside* this
                 buffer, so an all-gather only has to pull the W-1 foreign regions from the peers' buffers;
* ``gfull_all``  the fp32 full-size gradient accumulators, from which each peer pulls and sums its slice;
* ``ctrl``       int32 words: ``[0]`` parameter epoch, ``[1+u]`` gradient epoch of unit ``u``, the ready / done words of
                 the streamed gradient slots, then the slot area of the scalar all-reduce.

In the *sharded* schedule (see :mod:`olmo_b200.parallel.fsdp`) the units that hold transformer blocks are not kept
gathered.  For those units a rank keeps only

* ``lowp_all``   its own compute-dtype shards, in symmetric memory, which peers gather from;
* ``full_slots`` two local buffers of the largest streamed unit's size that gathered units rotate through;
* ``gslots``     three full-size fp32 gradient buffers in symmetric memory that the units rotate through in the backward
                 pass, each guarded by a *ready* word (this rank has finished writing use ``q``) and a *done* word (this
                 rank has finished reading use ``q`` from every peer).

Ordering protocol (all flags are monotone epochs, all waits bounded):

* after its optimizer step a rank publishes ``param_epoch``; a peer's all-gather reads that rank's shard only once the
  epoch has arrived;
* after the last micro-batch's backward pass of a unit a rank publishes ``grad_epoch[u]``; a peer reduces its slice of
  unit ``u`` only once every rank has published it;
* the scalar all-reduce of Σg² at the end of the step is also the barrier that makes it safe to overwrite shards and
  zero gradient accumulators for the next step: no rank gets past it before every rank has finished its reads.
"""
from __future__ import annotations

import ctypes
import logging
import os
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops import check, lib, ptr, status_tensor, stream_ptr

__all__ = ["CommTask", "PeerComm", "COMM_ALL_GATHER", "COMM_REDUCE_SCATTER"]

log = logging.getLogger(__name__)

COMM_NONE, COMM_ALL_GATHER, COMM_REDUCE_SCATTER = 0, 1, 2
MAX_WORLD = 8


class CommTask(ctypes.Structure):
    """Mirror of ``ob::CommTask`` (csrc/comm.cuh)."""

    _fields_ = [
        ("kind", ctypes.c_int),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("wait_value", ctypes.c_int),
        ("elems", ctypes.c_longlong),
        ("dst_peer_stride", ctypes.c_longlong),
        ("src", ctypes.c_void_p * MAX_WORLD),
        ("wait_flags", ctypes.c_void_p * MAX_WORLD),
        ("dst", ctypes.c_void_p),
        ("scale", ctypes.c_float),
        ("sumsq_partials", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("wait_cycles", ctypes.c_longlong),
        ("mode", ctypes.c_int),
        ("reserved", ctypes.c_int),
    ]


COMM_MODE_SELF, COMM_MODE_STORE = 2, 4
N_GSLOTS, N_FULL_SLOTS = 3, 2


#: how a unit's collective is divided over the four GEMMs of a block, in sixteenths, proportional to GEMM duration at
#: the 7B shapes (att_proj 0.55 ms, attn_out 0.18 ms, ff_proj 1.04 ms, ff_out 0.62 ms; same for the input-gradient GEMMs)
FWD_SPANS = {"att_proj": (0, 4, 16), "attn_out": (4, 5, 16), "ff_proj": (5, 12, 16), "ff_out": (12, 16, 16)}
BWD_SPANS = {"ff_out_dgrad": (0, 4, 16), "ff_proj_dgrad": (4, 11, 16), "attn_out_dgrad": (11, 12, 16), "att_proj_dgrad": (12, 16, 16)}
#: the same division over the four weight-gradient GEMMs of a block (they carry the backward pass's re-gather)
WGRAD_SPANS = {"ff_out": (0, 4, 16), "ff_proj": (4, 11, 16), "attn_out": (11, 12, 16), "att_proj": (12, 16, 16)}


class PeerComm:
    def __init__(self, engine, group) -> None:
        # These kernels only use plain peer loads and stores.  Asking torch not to bind the buffers to an NVLink multicast
        # object (best effort: the variable is ignored by releases that do not know it) keeps a rank that dies from
        # disturbing its peers through such a binding.
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem

        self.engine = engine
        # `world` / `rank` are those of the shard group (what gathers and reduce-scatters run over).  The buffers are
        # exchanged over the whole job, so a rank also knows the pointers of its replica group: the ranks that hold the
        # same shard in the other model replicas (hybrid sharding; plain data parallelism is a shard group of one).
        self.world, self.rank = engine.shard_world, engine.shard_rank
        self.gworld = getattr(engine, "world", self.world)
        self.grank = getattr(engine, "rank", self.rank)
        self.replicas = self.gworld // self.world
        assert self.gworld <= MAX_WORLD and self.world * self.replicas == self.gworld
        first = (self.grank // self.world) * self.world
        self.shard_peers = list(range(first, first + self.world))            # global ranks of my shard group, by shard rank
        self.replica_peers = list(range(self.rank, self.gworld, self.world))  # global ranks holding my shard, by replica
        self.replica_index = self.grank // self.world
        dev = engine.device
        assert ctypes.sizeof(CommTask) == lib().ob_comm_task_size(), "CommTask layout mismatch"
        # resident units: gathered copy and full-size gradient accumulator of every unit, end to end
        self.bases: List[int] = []
        off = 0
        for u in engine.units:
            self.bases.append(off)
            if not getattr(u, "streamed", False):
                off += u.numel
        total = max(off, 1024)
        self.full_all = symm_mem.empty(total, dtype=engine.compute_dtype, device=dev)
        self.h_full = symm_mem.rendezvous(self.full_all, group)
        self.gfull_all = symm_mem.empty(total, dtype=torch.float32, device=dev)
        self.h_gfull = symm_mem.rendezvous(self.gfull_all, group)
        # streamed units: own shards + rotating slots
        streamed = [u for u in engine.units if getattr(u, "streamed", False)]
        self.lowp_bases = {}
        off = 0
        for u in streamed:
            self.lowp_bases[u.index] = off
            off += u.shard_size
        self.slot_numel = max([u.numel for u in streamed], default=0)
        self.lowp_all = self.gslots = self.full_slots = None
        self.lowp_ptrs: List[int] = []
        self.gslot_ptrs: List[int] = []
        if streamed:
            self.lowp_all = symm_mem.empty(off, dtype=engine.compute_dtype, device=dev)
            self.h_lowp = symm_mem.rendezvous(self.lowp_all, group)
            self.gslots = symm_mem.empty(N_GSLOTS * self.slot_numel, dtype=torch.float32, device=dev)
            self.h_gslots = symm_mem.rendezvous(self.gslots, group)
            self.full_slots = torch.zeros(N_FULL_SLOTS * self.slot_numel, dtype=engine.compute_dtype, device=dev)
            self.lowp_all.zero_()
            self.gslots.zero_()
            self.lowp_ptrs = [int(self.h_lowp.buffer_ptrs[g]) for g in self.shard_peers]
            self.gslot_ptrs = [int(self.h_gslots.buffer_ptrs[g]) for g in self.shard_peers]
        # with model replicas, a reduce-scatter lands in a staging shard that the replica group then sums
        self.stage_all = None
        self.stage_bases: List[int] = []
        self.stage_ptrs: List[int] = []
        if self.replicas > 1:
            off = 0
            for u in engine.units:
                self.stage_bases.append(off)
                off += u.shard_size
            self.stage_all = symm_mem.empty(max(off, 1024), dtype=torch.float32, device=dev)
            self.h_stage = symm_mem.rendezvous(self.stage_all, group)
            self.stage_all.zero_()
            self.stage_ptrs = [int(self.h_stage.buffer_ptrs[g]) for g in self.replica_peers]
        self.n_units = len(engine.units)
        self.slot_words = lib().ob_scalar_slots_bytes() // 4
        self.gslot_word0 = 1 + self.n_units  # ready words of the gradient slots, then their done words
        self.stage_word0 = self.gslot_word0 + 2 * N_GSLOTS  # per unit: the staged (shard-group reduced) gradient is complete
        self.slot_off = (self.stage_word0 + self.n_units + 15) // 16 * 16
        self.ctrl = symm_mem.empty(self.slot_off + self.slot_words, dtype=torch.int32, device=dev)
        self.h_ctrl = symm_mem.rendezvous(self.ctrl, group)
        self.full_all.zero_()
        self.gfull_all.zero_()
        self.ctrl.zero_()
        self.full_ptrs = [int(self.h_full.buffer_ptrs[g]) for g in self.shard_peers]
        self.gfull_ptrs = [int(self.h_gfull.buffer_ptrs[g]) for g in self.shard_peers]
        self.ctrl_ptrs = [int(self.h_ctrl.buffer_ptrs[g]) for g in self.shard_peers]
        self.ctrl_ptrs_replica = [int(self.h_ctrl.buffer_ptrs[g]) for g in self.replica_peers]
        self.gslot_use = [0] * N_GSLOTS  # how often each gradient slot has been handed out (same on every rank)
        # the scalar all-reduce (and with it the end-of-step barrier) spans the whole job
        self.slot_ptrs_dev = torch.tensor([int(p) + 4 * self.slot_off for p in self.h_ctrl.buffer_ptrs], dtype=torch.int64, device=dev)
        self.param_epoch = 0
        self.grad_epoch = 0
        self.scalar_epoch = 0
        # How a GEMM launch carries a collective.  0 (default): the ten spare warps of every GEMM CTA move that CTA's
        # share, so no SM is taken from the GEMM.  An even number n > 0: the first n CTAs of the grid are set aside for
        # the collective instead (the two-CTA GEMM schedules CTA pairs).
        self.comm_ctas = int(os.environ.get("OLMO_B200_COMM_CTAS", "0"))
        self.rs_ctas = int(os.environ.get("OLMO_B200_RS_CTAS", "0"))
        self.standalone_ctas = int(os.environ.get("OLMO_B200_COMM_STANDALONE_CTAS", "64"))
        ms = float(os.environ.get("OLMO_B200_WAIT_BUDGET_MS", "30000"))
        self.wait_cycles = int(ms * 1.9e6)
        self._scalar_out = torch.zeros(1, dtype=torch.float32, device=dev)
        # Σg² of what the reduce-scatter kernels add to the local shards, one slot per communication CTA: the gradient
        # norm then needs no separate pass over the shards (OLMO_B200_RS_SUMSQ=0 restores the separate pass)
        self.fuse_sumsq = os.environ.get("OLMO_B200_RS_SUMSQ", "1").strip().lower() not in ("0", "false", "no", "off")
        self.rs_partials = torch.zeros(256, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        dist.barrier(group=group)
        self.group = group

    @classmethod
    def create(cls, engine) -> Optional["PeerComm"]:
        """Peer memory needs every rank of the job on one NVLink domain: at most eight ranks, all on this node."""
        from ..torch_util import get_local_world_size

        if engine.world > MAX_WORLD or get_local_world_size() != engine.world:
            log.info("the job spans more than one node (or more than %d ranks): collectives go through NCCL", MAX_WORLD)
            return None
        return cls(engine, dist.group.WORLD)

    # ------------------------------------------------------------------------------- buffers
    def full_view(self, unit_index: int, numel: int) -> torch.Tensor:
        b = self.bases[unit_index]
        return self.full_all[b : b + numel]

    def gfull_view(self, unit_index: int, numel: int) -> torch.Tensor:
        b = self.bases[unit_index]
        return self.gfull_all[b : b + numel]

    def lowp_view(self, unit) -> torch.Tensor:
        b = self.lowp_bases[unit.index]
        return self.lowp_all[b : b + unit.shard_size]

    def full_slot(self, slot: int) -> torch.Tensor:
        return self.full_slots[slot * self.slot_numel : (slot + 1) * self.slot_numel]

    def gslot(self, slot: int) -> torch.Tensor:
        return self.gslots[slot * self.slot_numel : (slot + 1) * self.slot_numel]

    # --------------------------------------------------------------------------------- tasks
    def _base_task(self, kind: int) -> CommTask:
        t = CommTask()
        t.kind, t.world, t.rank = kind, self.world, self.rank
        t.status = status_tensor(self.engine.device).data_ptr()
        t.wait_cycles = self.wait_cycles
        t.sumsq_partials = None
        t.mode = 0
        return t

    @staticmethod
    def _slice(S: int, part: int, parts: int, span, align: int):
        """``[a, b)`` of a shard of ``S`` elements: either part ``part`` of ``parts`` or ``span = (lo, hi, denominator)``."""
        if span is not None:
            lo, hi, den = span
            a = (S * lo // den) // align * align
            b = S if hi == den else (S * hi // den) // align * align
            return a, b
        step = (S // parts) // align * align
        a = part * step
        return a, (S if part == parts - 1 else a + step)

    def ag_task(self, unit, part: int = 0, parts: int = 1, span=None) -> CommTask:
        """All-gather of one slice of every foreign shard of ``unit`` into the local ``full`` buffer."""
        S = unit.shard_size
        esz = self.full_all.element_size()
        a, b = self._slice(S, part, parts, span, 8)
        t = self._base_task(COMM_ALL_GATHER)
        t.elems, t.dst_peer_stride = b - a, S
        base = self.bases[unit.index]
        for p in range(self.world):
            t.src[p] = self.full_ptrs[p] + (base + p * S + a) * esz
            t.wait_flags[p] = self.ctrl_ptrs[p]  # word 0: that rank's parameter epoch
        t.dst = self.full_ptrs[self.rank] + (base + a) * esz
        t.wait_value = self.param_epoch
        return t

    def rs_task(self, unit, part: int = 0, parts: int = 1, span=None) -> CommTask:
        """Reduce-scatter of one slice of this rank's gradient shard of ``unit`` (sum over ranks, scaled, added)."""
        S = unit.shard_size
        a, b = self._slice(S, part, parts, span, 4)
        t = self._base_task(COMM_REDUCE_SCATTER)
        t.elems = b - a
        base = self.bases[unit.index]
        for p in range(self.world):
            t.src[p] = self.gfull_ptrs[p] + (base + self.rank * S + a) * 4
            t.wait_flags[p] = self.ctrl_ptrs[p] + 4 * (1 + unit.index)
        t.scale = 1.0 / self.engine.world
        t.wait_value = self.grad_epoch
        if self.replicas > 1:  # lands in the staging shard (plain store); the replica group sums it into `grad` afterwards
            t.dst = self.stage_all.data_ptr() + (self.stage_bases[unit.index] + a) * 4
            t.mode |= COMM_MODE_STORE
            return t
        t.dst = unit.grad.data_ptr() + a * 4
        if self.fuse_sumsq:
            t.sumsq_partials = self.rs_partials.data_ptr()
        return t

    def replica_task(self, unit) -> CommTask:
        """Sum of the staged shard of ``unit`` over the replica group (every replica reads all of them, in replica order,
        so all end up with bit-identical gradients), added to the fp32 gradient shard, with its Σg²."""
        t = CommTask()
        t.kind, t.world, t.rank = COMM_REDUCE_SCATTER, self.replicas, self.replica_index
        t.status = status_tensor(self.engine.device).data_ptr()
        t.wait_cycles = self.wait_cycles
        t.mode = 0
        t.elems = unit.shard_size
        for k in range(self.replicas):
            t.src[k] = self.stage_ptrs[k] + self.stage_bases[unit.index] * 4
            t.wait_flags[k] = self.ctrl_ptrs_replica[k] + 4 * (self.stage_word0 + unit.index)
        t.dst = unit.grad.data_ptr()
        t.sumsq_partials = self.rs_partials.data_ptr() if self.fuse_sumsq else None
        t.scale = 1.0
        t.wait_value = self.grad_epoch
        return t

    def finish_replicas(self, unit) -> None:
        """Call once the reduce-scatter of ``unit`` has been enqueued on this stream: publish the staged shard and add
        the replica group's sum to the gradient shard."""
        if self.replicas > 1:
            self.signal(self.stage_word0 + unit.index, self.grad_epoch)
            self.launch(self.replica_task(unit))

    def stream_ag_task(self, unit, slot: int, span=None) -> CommTask:
        """Gather of one slice of every rank's shard of a streamed ``unit`` (this rank's own included) into local
        full-size slot ``slot``."""
        S = unit.shard_size
        esz = self.lowp_all.element_size()
        a, b = self._slice(S, 0, 1, span, 8)
        t = self._base_task(COMM_ALL_GATHER)
        t.mode |= COMM_MODE_SELF
        t.elems, t.dst_peer_stride = b - a, S
        base = self.lowp_bases[unit.index]
        for p in range(self.world):
            t.src[p] = self.lowp_ptrs[p] + (base + a) * esz
            t.wait_flags[p] = None if p == self.rank else self.ctrl_ptrs[p]
        t.dst = self.full_slots.data_ptr() + (slot * self.slot_numel + a) * esz
        t.wait_value = self.param_epoch
        return t

    def stream_rs_task(self, unit, gslot: int, span=None, with_sumsq: bool = False) -> CommTask:
        """Reduce-scatter of one slice of this rank's shard of a streamed ``unit`` out of every rank's gradient slot
        ``gslot``, added to the fp32 gradient shard.  Waits for use ``gslot_use[gslot]`` of the slot to be ready."""
        S = unit.shard_size
        a, b = self._slice(S, 0, 1, span, 4)
        t = self._base_task(COMM_REDUCE_SCATTER)
        t.elems = b - a
        for p in range(self.world):
            t.src[p] = self.gslot_ptrs[p] + (gslot * self.slot_numel + self.rank * S + a) * 4
            t.wait_flags[p] = self.ctrl_ptrs[p] + 4 * (self.gslot_word0 + gslot)
        t.dst = unit.grad.data_ptr() + a * 4
        if with_sumsq and self.fuse_sumsq:
            t.sumsq_partials = self.rs_partials.data_ptr()
        t.scale = 1.0 / self.engine.world
        t.wait_value = self.gslot_use[gslot]
        return t

    def open_gslot(self, gslot: int) -> int:
        """Hand out gradient slot ``gslot`` for its next use: first wait (on the stream, bounded) until every peer has
        finished reading the previous use.  Returns the new use number."""
        prev = self.gslot_use[gslot]
        if prev > 0:
            word = self.gslot_word0 + N_GSLOTS + gslot
            flags = (ctypes.c_void_p * MAX_WORLD)()
            for p in range(self.world):
                flags[p] = None if p == self.rank else self.ctrl_ptrs[p] + 4 * word
            check(lib().ob_wait_flags(flags, ctypes.c_int(self.world), ctypes.c_int(prev), ptr(status_tensor(self.engine.device)),
                                      ctypes.c_longlong(self.wait_cycles), stream_ptr()), "ob_wait_flags")
        self.gslot_use[gslot] = prev + 1
        return prev + 1

    def publish_gslot(self, gslot: int) -> None:
        """This rank's gradients of the slot's current use are complete."""
        self.signal(self.gslot_word0 + gslot, self.gslot_use[gslot])

    def release_gslot(self, gslot: int) -> None:
        """This rank has finished reading the slot's current use from every peer."""
        self.signal(self.gslot_word0 + N_GSLOTS + gslot, self.gslot_use[gslot])

    # ------------------------------------------------------------------------------ launches
    def launch(self, task: CommTask, ctas: Optional[int] = None) -> None:
        n = ctas or self.standalone_ctas
        assert n <= self.rs_partials.numel()
        check(lib().ob_comm_launch(ctypes.byref(task), ctypes.c_int(n), stream_ptr()), "ob_comm_launch")

    def signal(self, word: int, value: int) -> None:
        check(lib().ob_signal(ctypes.c_void_p(self.ctrl_ptrs[self.rank] + 4 * word), ctypes.c_int(value), stream_ptr()), "ob_signal")

    def publish_params(self) -> None:
        """Call after the optimizer step has been enqueued: peers may now read this rank's shards."""
        self.param_epoch += 1
        self.signal(0, self.param_epoch)

    def begin_grad_epoch(self) -> None:
        self.grad_epoch += 1

    def publish_grads(self, unit) -> None:
        self.signal(1 + unit.index, self.grad_epoch)

    def all_gather_units(self, units: Sequence) -> None:
        for u in units:
            self.launch(self.ag_task(u))

    def reduce_scatter_units(self, units: Sequence, scale: float) -> None:
        del scale  # tasks carry 1/world
        for u in units:
            self.launch(self.rs_task(u))

    def all_reduce_scalar_(self, value: torch.Tensor) -> torch.Tensor:
        """In-place sum of a one-element fp32 tensor over the shard group (computed as the sum over the whole job divided
        by the number of replicas, which all hold the same values); also an execution barrier of the whole job on the stream."""
        self.scalar_epoch += 1
        rc = lib().ob_allreduce_scalar(
            ptr(value), ptr(self.slot_ptrs_dev), ctypes.c_void_p(self.ctrl_ptrs[self.rank] + 4 * self.slot_off), ptr(self._scalar_out),
            ctypes.c_int(self.grank), ctypes.c_int(self.gworld), ctypes.c_int(self.scalar_epoch),
            ptr(status_tensor(self.engine.device)), ctypes.c_longlong(self.wait_cycles), stream_ptr(),
        )
        check(rc, "ob_allreduce_scalar")
        value.copy_(self._scalar_out)
        if self.replicas > 1:  # every replica contributed the same per-shard values
            value.div_(self.replicas)
        return value
