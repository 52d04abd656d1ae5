"""Multi-process CPU tests over gloo: sharded training equals single-process training, checkpoints re-shard across
world sizes, cancellation is agreed on by all ranks, and a rank that disappears surfaces as an error on the others."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

WORKER = Path(__file__).resolve().parent / "dist_cpu_worker.py"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(nproc: int, scenario: str, out: Path, work: Path, *extra: str, expect_ok: bool = True, timeout: int = 600):
    work.mkdir(parents=True, exist_ok=True)
    env = dict(os.environ, OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")
    args = [str(WORKER), scenario, "--out", str(out), "--work", str(work), *extra]
    if nproc == 1:
        cmd = [sys.executable, *args]
    else:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1",
               "--master-port", str(_free_port()), *args]
    proc = subprocess.run(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=timeout)
    if expect_ok:
        assert proc.returncode == 0, proc.stdout[-5000:]
        return torch.load(out, weights_only=False)
    return proc


def assert_same_training(a, b, what, tol=5e-5):
    for x, y in zip(a["steps"], b["steps"]):
        assert abs(x["loss"] - y["loss"]) < 1e-4, f"{what}: {a['steps']} vs {b['steps']}"
        assert abs(x["norm"] - y["norm"]) < 1e-3 * max(1.0, y["norm"]), f"{what}: {a['steps']} vs {b['steps']}"
    for name, t in a["state"].items():
        torch.testing.assert_close(t, b["state"][name], rtol=1e-4, atol=tol, msg=lambda m: f"{what}: {name}: {m}")


@pytest.fixture(scope="module")
def single(tmp_path_factory):
    d = tmp_path_factory.mktemp("single")
    return launch(1, "train", d / "one.pt", d / "work")


@pytest.mark.parametrize(
    "nproc,extra",
    [
        (2, ("--wrap", "by_block_and_size")),
        (2, ("--strategy", "NO_SHARD")),
        (4, ("--strategy", "HYBRID_SHARD", "--replicas", "2")),
    ],
)
def test_sharded_training_matches_single_process(tmp_path, single, nproc, extra):
    multi = launch(nproc, "train", tmp_path / "multi.pt", tmp_path / "work", *extra)
    assert multi["world"] == nproc
    assert_same_training(multi, single, f"{nproc} ranks {extra}")


def test_lion_sharded_matches_single(tmp_path):
    one = launch(1, "train", tmp_path / "one.pt", tmp_path / "w1", "--optimizer", "lionw")
    two = launch(2, "train", tmp_path / "two.pt", tmp_path / "w2", "--optimizer", "lionw")
    assert_same_training(two, one, "lion 2 ranks", tol=5e-3)  # sign updates amplify last-bit differences


@pytest.mark.parametrize("checkpointer", ["olmo_core"])
def test_checkpoint_resharding_across_world_sizes(tmp_path, checkpointer):
    saved = launch(2, "save", tmp_path / "saved.pt", tmp_path / "run", "--checkpointer", checkpointer)
    sharded, unsharded = Path(saved["sharded"]), Path(saved["unsharded"])
    assert (sharded / "config.yaml").is_file() and (unsharded / "config.yaml").is_file()
    assert (unsharded / "model.safetensors").is_file() or (unsharded / "model.pt").is_file()

    # same world size, fewer ranks, and the unsharded checkpoint all restore the same weights and the same next step
    for nproc, load in ((1, sharded), (4, sharded), (2, unsharded)):
        got = launch(nproc, "restore", tmp_path / f"r{nproc}_{load.name}.pt", tmp_path / f"w{nproc}_{load.name}", "--load", str(load),
                     "--checkpointer", checkpointer, "--force-fsdp")
        assert got["global_step"] == 3
        for name, t in got["state"].items():
            torch.testing.assert_close(t, saved["state"][name], rtol=0, atol=0, msg=lambda m: f"{nproc} ranks from {load.name}: {name}: {m}")
        assert abs(got["next"][0]["loss"] - saved["next"][0]["loss"]) < 1e-4, (nproc, load.name)

    # offline conversion: sharded directory -> full tensors, no process group
    from olmo_b200.checkpoint import build_sharded_checkpointer
    from olmo_b200.config import TrainConfig

    cfg = TrainConfig.load(sharded / "config.yaml", validate_paths=False)
    model_state, optim_state, trainer_state = build_sharded_checkpointer(cfg).unshard_checkpoint(sharded)
    for name, t in saved["state"].items():
        torch.testing.assert_close(model_state[name], t, rtol=0, atol=0)
    assert trainer_state["global_step"] == 3
    assert optim_state is not None and len(optim_state["state"]) == len(saved["state"])

    # the unsharded optimizer file must carry every parameter, including those whose shard on rank 0 is empty (the
    # per-parameter optimizer keeps no state for an empty shard), with the step count and moments of the sharded one
    full_optim = torch.load(unsharded / "optim.pt", map_location="cpu", weights_only=False)
    assert set(full_optim["state"]) == set(saved["state"])
    for name, st in full_optim["state"].items():
        assert int(st["step"]) == 3, (name, st["step"])
        for key in ("exp_avg", "exp_avg_sq"):
            torch.testing.assert_close(st[key], optim_state["state"][name][key], rtol=0, atol=0, msg=lambda m: f"{name}.{key}: {m}")


def test_reference_torch_new_layout_is_written_by_two_ranks_and_read_by_one(tmp_path, monkeypatch):
    """Two ranks write their sharded checkpoint in the reference's ``torch_new`` layout (full tensors gathered to rank 0,
    one trainer-state file per rank); one rank and two ranks resume from it with the saved weights and the same next loss."""
    from olmo_b200.checkpoint_compat import detect_layout

    monkeypatch.setenv("OLMO_B200_WRITE_REFERENCE_LAYOUT", "1")
    saved = launch(2, "save", tmp_path / "saved.pt", tmp_path / "run", "--checkpointer", "torch_new")
    sharded = Path(saved["sharded"])
    assert detect_layout(sharded) == "torch_new" and (sharded / "train" / "rank1.pt").is_file()
    for nproc in (1, 2):
        got = launch(nproc, "restore", tmp_path / f"r{nproc}.pt", tmp_path / f"w{nproc}", "--load", str(sharded), "--checkpointer", "torch_new",
                     "--force-fsdp")
        assert got["global_step"] == 3
        for name, t in got["state"].items():
            torch.testing.assert_close(t, saved["state"][name], rtol=0, atol=0, msg=lambda m: f"{nproc} ranks: {name}: {m}")
        assert abs(got["next"][0]["loss"] - saved["next"][0]["loss"]) < 1e-4, nproc


def test_all_ranks_agree_on_cancellation(tmp_path):
    got = launch(2, "cancel", tmp_path / "c.pt", tmp_path / "w", "--time-limit", "100")
    assert got["stopped_at"] == 1


def test_lost_rank_is_reported_not_hung(tmp_path):
    out = tmp_path / "lost.pt"
    proc = launch(2, "lost_rank", out, tmp_path / "w", "--pg-timeout", "8", expect_ok=False, timeout=300)
    survivor = torch.load(f"{out}.rank0", weights_only=False)
    assert torch.load(f"{out}.rank1", weights_only=False)["left"]
    assert survivor["error"] is not None, proc.stdout[-3000:]
    assert survivor["waited"] < 60


# ------------------------------------------------------------------------------ host-side checkpoint faults


def test_rank_lost_during_a_save_leaves_no_half_written_checkpoint(tmp_path):
    """The save protocol writes into ``step{N}-tmp`` and renames after every rank has finished
    (reference: ``olmo/checkpoint.py:550-603``).  A rank that dies between its shard write and the rename must leave
    the earlier checkpoint as the latest valid one and no ``step3`` folder at all."""
    proc = launch(2, "save_crash", tmp_path / "crash.pt", tmp_path / "run", "--pg-timeout", "20", expect_ok=False, timeout=300)
    assert proc.returncode != 0
    info = torch.load(tmp_path / "crash.pt", weights_only=False)
    run = tmp_path / "run"
    assert Path(info["good"]).name == "step2" and (run / "step2" / "metadata.yaml").is_file()
    assert not (run / "step3").exists(), sorted(p.name for p in run.iterdir())
    assert (run / "step3-tmp").is_dir()  # what was written stays out of the way under the temporary name
    assert (run / "latest").resolve().name == "step2"
    survivor = torch.load(f"{tmp_path / 'crash.pt'}.rank0", weights_only=False)
    assert survivor["error"]  # rank 0 got an exception from the barrier, it did not hang
    # and a new job resumes from the good one
    got = launch(2, "restore", tmp_path / "resume.pt", tmp_path / "w2", "--load", str(run / "step2"), "--force-fsdp")
    assert got["global_step"] == 2


def _saved_two_rank_checkpoint(tmp_path) -> Path:
    saved = launch(2, "save", tmp_path / "saved.pt", tmp_path / "run")
    return Path(saved["sharded"])


def test_truncated_and_missing_shard_files_stop_the_restore(tmp_path):
    import shutil

    from olmo_b200.checkpoint import build_sharded_checkpointer
    from olmo_b200.config import TrainConfig
    from olmo_b200.exceptions import OLMoCheckpointError

    good = _saved_two_rank_checkpoint(tmp_path)
    cfg = TrainConfig.load(good / "config.yaml", validate_paths=False)

    cut = tmp_path / "cut"
    shutil.copytree(good, cut)
    victim = cut / "model" / "rank1.pt"
    victim.write_bytes(victim.read_bytes()[: victim.stat().st_size // 2])
    with pytest.raises(OLMoCheckpointError, match="rank1.pt.*(truncated|corrupt)"):
        build_sharded_checkpointer(cfg).unshard_checkpoint(cut)
    proc = launch(2, "restore", tmp_path / "r_cut.pt", tmp_path / "w_cut", "--load", str(cut), "--force-fsdp", "--pg-timeout", "20", expect_ok=False, timeout=300)
    assert proc.returncode != 0 and "truncated or corrupt" in proc.stdout

    gone = tmp_path / "gone"
    shutil.copytree(good, gone)
    (gone / "optim" / "rank0.pt").unlink()
    with pytest.raises(FileNotFoundError, match="rank0.pt"):
        build_sharded_checkpointer(cfg).unshard_checkpoint(gone)
    # the weights alone are still readable
    model_state, optim_state, _ = build_sharded_checkpointer(cfg).unshard_checkpoint(gone, load_optimizer_state=False)
    assert optim_state is None and len(model_state) > 0
