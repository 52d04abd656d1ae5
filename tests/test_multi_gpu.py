"""Multi-GPU equivalence: N ranks with peer-memory collectives (and with NCCL collectives) reach the same weights as a
single GPU that processes the same global batch.  Needs at least two GPUs; ranks run as child processes."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).resolve().parent / "multi_gpu_worker.py"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(nproc: int, out: Path, *extra: str) -> dict:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if nproc == 1:
        cmd = [sys.executable, str(WORKER), "--out", str(out), *extra]
    else:
        cmd = [
            sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
            "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(WORKER), "--out", str(out), *extra,
        ]
    proc = subprocess.run(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-4000:]
    return torch.load(out, weights_only=False)


def _compare(a: dict, b: dict, what: str) -> None:
    for x, y in zip(a["norms"], b["norms"]):
        assert abs(x - y) <= 2e-2 * abs(y) + 1e-6, f"{what}: grad norms {a['norms']} vs {b['norms']}"
    for name, t in a["state"].items():
        r = b["state"][name]
        err = (t - r).abs().max().item()
        assert err <= 2e-3 + 2e-2 * r.abs().max().item(), f"{what}: {name} differs by {err}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fused_comm", [1, 0])
def test_two_ranks_match_one(tmp_path, fused_comm):
    single = _run(1, tmp_path / "one.pt")
    multi = _run(2, tmp_path / f"two_{fused_comm}.pt", "--fused-comm", str(fused_comm))
    _compare(multi, single, f"2 ranks (fused_comm={fused_comm}) vs 1")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("comm_ctas", [0, 8])
def test_sharded_schedule_matches_one(tmp_path, comm_ctas):
    """The FULL_SHARD schedule proper (block units streamed through parameter and gradient slots, a gather in forward and
    in backward and a reduce-scatter per micro-batch, all riding on block GEMMs) against one GPU on the same batch."""
    single = _run(1, tmp_path / "one.pt", "--layers", "5")
    multi = _run(2, tmp_path / f"sharded_{comm_ctas}.pt", "--schedule", "sharded", "--layers", "5", "--comm-ctas", str(comm_ctas))
    _compare(multi, single, f"2 ranks sharded schedule (comm_ctas={comm_ctas}) vs 1")
    assert abs(multi["eval_ce"] - multi["module_ce"]) < 2e-2 * abs(multi["module_ce"]), (multi["eval_ce"], multi["module_ce"])
    assert abs(multi["eval_ce"] - single["eval_ce"]) < 2e-2 * abs(single["eval_ce"])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_schedule_with_activation_checkpointing(tmp_path):
    single = _run(1, tmp_path / "one.pt", "--layers", "4", "--activation-checkpointing", "whole_layer")
    multi = _run(2, tmp_path / "sharded_ac.pt", "--schedule", "sharded", "--layers", "4", "--activation-checkpointing", "whole_layer")
    _compare(multi, single, "2 ranks sharded schedule + whole_layer checkpointing vs 1")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("schedule", ["resident", "sharded"])
def test_fused_collectives_are_reproducible(tmp_path, schedule):
    """Peers are summed in rank order and every partial sum has one writer, so two runs from the same seed must give
    bit-identical weights and gradient norms."""
    a = _run(2, tmp_path / "a.pt", "--schedule", schedule, "--layers", "4")
    b = _run(2, tmp_path / "b.pt", "--schedule", schedule, "--layers", "4")
    assert a["norms"] == b["norms"]
    for name, t in a["state"].items():
        assert torch.equal(t, b["state"][name]), name


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("schedule", ["resident", "sharded"])
def test_sharded_checkpoint_resume_is_exact(tmp_path, schedule):
    """A run that saves a sharded checkpoint after its second step, loses its weights and optimizer moments and restores
    them ends with the same bits as an uninterrupted run (gathered copies and streamed shards are refreshed on restore)."""
    plain = _run(2, tmp_path / "a.pt", "--schedule", schedule, "--layers", "4", "--steps", "4")
    (tmp_path / "ckpt").mkdir()
    resumed = _run(2, tmp_path / "b.pt", "--schedule", schedule, "--layers", "4", "--steps", "4", "--resume-at", "2", "--ckpt-dir", str(tmp_path / "ckpt"))
    assert plain["norms"] == resumed["norms"]
    for name, t in plain["state"].items():
        assert torch.equal(t, resumed["state"][name]), name


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_replicated_data_parallel_on_peer_memory_matches_one(tmp_path):
    """NO_SHARD (what ``ddp`` maps to): a shard group of one, gradients summed over the replica group by the peer-memory
    kernel (the worker asserts that the peer-memory runtime is active)."""
    single = _run(1, tmp_path / "one.pt")
    multi = _run(2, tmp_path / "ddp.pt", "--strategy", "NO_SHARD")
    _compare(multi, single, "2 replicas vs 1")


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_hybrid_shard_matches_one(tmp_path):
    """HYBRID_SHARD, two replicas of two shards: reduce-scatter inside the shard group into a staging shard, then the
    replica group's sum, both through peer memory (the worker asserts ``engine.comm is not None``)."""
    single = _run(1, tmp_path / "one.pt")
    multi = _run(4, tmp_path / "hybrid.pt", "--strategy", "HYBRID_SHARD", "--replicas", "2")
    _compare(multi, single, "4 ranks hybrid vs 1")
    again = _run(4, tmp_path / "hybrid2.pt", "--strategy", "HYBRID_SHARD", "--replicas", "2")
    assert again["norms"] == multi["norms"] and all(torch.equal(t, multi["state"][n]) for n, t in again["state"].items())
