"""Book-keeping of the sharded (FULL_SHARD) schedule, driven on the CPU against a recording stand-in for the peer-memory
runtime: which unit sits in which parameter slot when a block uses it, what is gathered stand-alone and what rides on
GEMMs, and that every streamed unit's gradients are published and reduced exactly once per micro-batch through a
gradient slot that is not handed out again before its reduction was launched."""
from types import SimpleNamespace

import pytest
import torch

from olmo_b200.parallel.fsdp import ParamSlot, Unit, _StreamState
from olmo_b200.parallel.peer import BWD_SPANS, FWD_SPANS, N_FULL_SLOTS, N_GSLOTS, WGRAD_SPANS


class FakeComm:
    def __init__(self, slot_numel):
        self.param_epoch = 0
        self.comm_ctas = self.rs_ctas = 0
        self.slot_numel = slot_numel
        self.full_slots = torch.zeros(N_FULL_SLOTS * slot_numel)
        self.gslots = torch.zeros(N_GSLOTS * slot_numel)
        self.log = []
        self.slot_holds = [None] * N_FULL_SLOTS    # what a gather (stand-alone or riding) last put into each parameter slot
        self.gslot_state = ["free"] * N_GSLOTS       # free -> open -> published -> reducing -> free

    def full_slot(self, s):
        return self.full_slots[s * self.slot_numel:(s + 1) * self.slot_numel]

    def gslot(self, s):
        return self.gslots[s * self.slot_numel:(s + 1) * self.slot_numel]

    def stream_ag_task(self, unit, slot, span=None):
        return ("ag", unit.stream_pos, slot, span)

    def stream_rs_task(self, unit, gslot, span=None, with_sumsq=False):
        return ("rs", unit.stream_pos, gslot, span, with_sumsq)

    def launch(self, task):
        self.run(task)
        self.log.append(("standalone",) + task)

    def run(self, task):  # what a kernel carrying `task` does to the buffers
        if task[0] == "ag":
            self.slot_holds[task[2]] = (task[1], self.param_epoch)
        else:
            assert self.gslot_state[task[2]] in ("published", "reducing"), (task, self.gslot_state)
            self.gslot_state[task[2]] = "reducing"

    def open_gslot(self, g):
        assert self.gslot_state[g] == "free", f"gradient slot {g} handed out while {self.gslot_state[g]}"
        self.gslot_state[g] = "open"

    def publish_gslot(self, g):
        assert self.gslot_state[g] == "open"
        self.gslot_state[g] = "published"

    def release_gslot(self, g):
        assert self.gslot_state[g] == "reducing"
        self.gslot_state[g] = "free"
        self.log.append(("released", g))


def make_state(n_blocks: int, blocks_per_unit: int = 1):
    units, blocks = [], []
    keys = ("att_proj", "attn_out", "ff_proj", "ff_out", "attn_norm", "ff_norm")
    for u in range(n_blocks // blocks_per_unit):
        slots, off = [], 0
        for b in range(blocks_per_unit):
            for k in keys:
                shape = torch.Size((8, 8)) if "norm" not in k else torch.Size((8,))
                numel = 64 if "norm" not in k else 8
                slots.append(ParamSlot(f"transformer.blocks.{u * blocks_per_unit + b}.{k}.weight", shape, numel, off, None, "weight"))
                off += 64
        unit = Unit(f"u{u}", u, slots, off, off // 2, streamed=True, stream_pos=u)
        unit.zero_ranges = [(sl.offset, sl.offset + 64) for sl in slots if len(sl.shape) == 1]
        units.append(unit)
        for b in range(blocks_per_unit):
            mods = {}
            for k in keys:
                sl = slots[b * len(keys) + keys.index(k)]
                w = SimpleNamespace(_ob_unit=unit, _ob_slot=sl)
                mods[k] = SimpleNamespace(weight=w)
            blocks.append(SimpleNamespace(q_norm=None, k_norm=None, **mods))
    comm = FakeComm(max(u.numel for u in units))
    engine = SimpleNamespace(units=units, comm=comm, model=SimpleNamespace(all_blocks=lambda: blocks))
    return _StreamState(engine), comm, len(blocks)


def run_microbatch(st, comm, n_blocks, is_last):
    """The call sequence of ``FlatShardEngine._train_microbatch_streamed`` with the kernels replaced by their effect."""
    n_stream = len(st.seq)

    def carry(kwargs):
        for kw in (kwargs or {}).values():
            comm.run(kw["comm"][0])
            comm.log.append(("riding",) + kw["comm"][0])

    for i in range(n_blocks):
        pos = st.block_pos[i]
        st.ensure(pos)
        gk = st.prefetch(pos + 1, FWD_SPANS) if st.last_block[pos] == i and pos + 1 < n_stream else None
        st.weights(i)
        assert comm.slot_holds[pos % N_FULL_SLOTS] == (pos, comm.param_epoch), f"forward of block {i} would read stale weights"
        carry(gk)
    for i in range(n_blocks - 1, -1, -1):
        pos = st.block_pos[i]
        st.ensure(pos)
        assert comm.slot_holds[pos % N_FULL_SLOTS] == (pos, comm.param_epoch), f"backward of block {i} would read stale weights"
        if st.last_block[pos] == i:
            st.open_grads(pos)
        wk = st.prefetch(pos - 1, WGRAD_SPANS) if st.first_block[pos] == i and pos - 1 >= 0 else None
        st.sink(i, wk)
        rk = st.rs_kwargs(BWD_SPANS, is_last)
        carry(wk)
        carry(rk)
        st.rs_done()
        if st.first_block[pos] == i:
            st.publish_grads(pos, is_last)
    st.flush_rs(is_last)


@pytest.mark.parametrize("n_blocks,per_unit", [(1, 1), (2, 1), (3, 1), (5, 1), (8, 1), (6, 2), (4, 4)])
def test_streamed_schedule_invariants(n_blocks, per_unit):
    st, comm, nb = make_state(n_blocks, per_unit)
    n_units = n_blocks // per_unit
    for step in range(2):
        for mb in range(3):
            comm.log.clear()
            run_microbatch(st, comm, nb, is_last=mb == 2)
            reduced = [e for e in comm.log if e[1] == "rs"]
            units_reduced = sorted({e[2] for e in reduced})
            assert units_reduced == list(range(n_units)), units_reduced   # every streamed unit, every micro-batch
            assert all(e[-1] == (mb == 2) for e in reduced)               # sum of squares only on the last micro-batch
            standalone_rs = [e for e in reduced if e[0] == "standalone"]
            assert {e[2] for e in standalone_rs} == {0}                   # only the first unit finds no GEMM to ride on
            assert all(s == "free" for s in comm.gslot_state)
            gathers = [e for e in comm.log if e[1] == "ag"]
            standalone_ag = [e for e in gathers if e[0] == "standalone"]
            if mb == 0:
                assert [e[2] for e in standalone_ag] == [0]               # only the first unit after new weights
            else:
                assert standalone_ag == []                                # everything else is prefetched or still in place
            riding_ag = {e[2] for e in gathers if e[0] == "riding"}
            if n_units > N_FULL_SLOTS:
                assert riding_ag                                          # gathers ride on forward and weight-gradient GEMMs
        comm.param_epoch += 1  # the optimizer step publishes new shards: every slot's content is stale
