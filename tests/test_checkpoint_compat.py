"""Sharded checkpoints in the reference implementation's own layouts are unsharded offline and can be resumed from."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch
import yaml

from olmo_b200.checkpoint_compat import (
    ShardedTensorRecord, detect_layout, load_with_sharded_tensor_records, unshard_local_checkpoint, unshard_reference_checkpoint,
    unshard_torch_legacy_checkpoint,
)
from olmo_b200.exceptions import OLMoCheckpointError

WORKER = Path(__file__).resolve().parent / "ref_layout_worker.py"
# names with FSDP's wrapper segment, as the reference writes them
NAMES = {
    "transformer.wte.weight": (10, 4),
    "transformer.blocks.0._fsdp_wrapped_module.att_proj.weight": (12, 4),
    "transformer.blocks.0._fsdp_wrapped_module.attn_norm.weight": (3,),  # fewer rows than ranks: a rank with no shard
    "transformer.ff_out.weight": (10, 4),
}


def _source(seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    model = {n: torch.randn(shape, generator=g) for n, shape in NAMES.items()}
    state = {n: {"exp_avg": torch.randn(shape, generator=g), "exp_avg_sq": torch.rand(shape, generator=g), "step": torch.tensor(7.0)}
             for n, shape in NAMES.items()}
    groups = [{"lr": 1e-3, "weight_decay": 0.1, "params": list(NAMES), "param_names": list(NAMES)}]
    return {"model": model, "optim": {"state": state, "param_groups": groups}, "trainer": {"global_step": 7, "epoch": 0}}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def legacy_dir(tmp_path_factory):
    root = tmp_path_factory.mktemp("legacy")
    torch.save(_source(), root / "source.pt")
    out = root / "step7"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=4", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(WORKER), "--source", str(root / "source.pt"), "--out", str(out)]
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=300, env=dict(os.environ))
    assert proc.returncode == 0, proc.stdout[-3000:]
    return out


def _clean(n):
    return n.replace("_fsdp_wrapped_module.", "")


def test_legacy_rank_file_unpickles_without_a_process_group(legacy_dir):
    state = load_with_sharded_tensor_records(legacy_dir / "rank1.pt")
    rec = state["model"]["transformer.wte.weight"]
    assert isinstance(rec, ShardedTensorRecord) and tuple(rec.size) == (10, 4)
    assert len(rec.metadata.shards_metadata) == 4 and len(rec.local_shards) == 1
    assert state["global_step"] == 7


def test_torch_legacy_checkpoint_unshards_to_the_full_tensors(legacy_dir):
    assert detect_layout(legacy_dir) == "torch_legacy"
    src = _source()
    model, optim, trainer = unshard_torch_legacy_checkpoint(legacy_dir)
    assert set(model) == {_clean(n) for n in NAMES}
    for n in NAMES:
        torch.testing.assert_close(model[_clean(n)], src["model"][n], rtol=0, atol=0)
        for key in ("exp_avg", "exp_avg_sq"):
            torch.testing.assert_close(optim["state"][_clean(n)][key], src["optim"]["state"][n][key], rtol=0, atol=0)
        assert float(optim["state"][_clean(n)]["step"]) == 7.0
    assert optim["param_groups"][0]["param_names"] == [_clean(n) for n in NAMES]
    assert trainer["global_step"] == 7 and "model" not in trainer and "optim" not in trainer
    model_only, no_optim, no_trainer = unshard_reference_checkpoint(legacy_dir, load_optimizer_state=False, load_trainer_state=False)
    assert no_optim is None and no_trainer is None and set(model_only) == set(model)


def test_torch_legacy_missing_rank_file_is_an_error(legacy_dir, tmp_path):
    import shutil

    broken = tmp_path / "broken"
    shutil.copytree(legacy_dir, broken)
    (broken / "rank3.pt").unlink()
    with pytest.raises(OLMoCheckpointError, match="missing|covered"):
        unshard_torch_legacy_checkpoint(broken)


def _write_local(folder: Path, src, world: int, old_torch: bool) -> None:
    """Hand-built ``local`` layout: the parameters laid end to end as one FSDP flat parameter per wrapped module, cut into
    ``world`` equal padded pieces, with the flat parameter's own tables in the form of torch >= 2.1 or <= 2.0."""
    from torch.distributed.fsdp._flat_param import _ShardParamInfo

    modules = {"": ["transformer.wte.weight", "transformer.ff_out.weight"],
               "transformer.blocks.0": ["transformer.blocks.0._fsdp_wrapped_module.att_proj.weight", "transformer.blocks.0._fsdp_wrapped_module.attn_norm.weight"]}
    ids = {n: i for i, n in enumerate(NAMES)}
    (folder / "model").mkdir(parents=True)
    (folder / "optim").mkdir()
    (folder / "train").mkdir()
    (folder / "metadata.yaml").write_text(yaml.safe_dump({"world_size": world}))
    per_rank_model = [{"modules": []} for _ in range(world)]
    per_rank_optim = [{"state": {}, "param_groups": [{"lr": 1e-3, "params": list(ids.values()), "param_names": list(NAMES)}]} for _ in range(world)]
    for prefix, names in modules.items():
        rel = [n[len(prefix) + 1:] if prefix else n for n in names]
        rel = [r.replace("_fsdp_wrapped_module.", "") for r in rel]
        flats = {key: torch.cat([t[n].reshape(-1) for n in names]) for key, t in
                 {"p": src["model"], "exp_avg": {n: src["optim"]["state"][n]["exp_avg"] for n in names},
                  "exp_avg_sq": {n: src["optim"]["state"][n]["exp_avg_sq"] for n in names}}.items()}
        total = flats["p"].numel()
        per = -(-total // world)
        starts, pos = [], 0
        for n in names:
            starts.append(pos)
            pos += src["model"][n].numel()
        for r in range(world):
            lo, hi = r * per, min((r + 1) * per, total)
            piece = torch.zeros(per)
            piece[: max(hi - lo, 0)] = flats["p"][lo:hi]
            infos, old_offsets, present = [], [], []
            for i, n in enumerate(names):
                a, b = max(starts[i], lo), min(starts[i] + src["model"][n].numel(), hi)
                if b > a:
                    infos.append(_ShardParamInfo(True, a - lo, b - a, a - starts[i], b - starts[i] - 1))
                    old_offsets.append((a - starts[i], b - starts[i] - 1))
                    present.append(i)
                    for key in ("exp_avg", "exp_avg_sq"):
                        per_rank_optim[r]["state"].setdefault(ids[n], {"step": torch.tensor(7.0)})[key] = flats[key][a:b].clone()
                else:
                    infos.append(_ShardParamInfo(False, None, None, None, None))
                    per_rank_optim[r]["state"].setdefault(ids[n], {"step": torch.tensor(7.0), "exp_avg": torch.empty(0), "exp_avg_sq": torch.empty(0)})
            handle = {"flat_param.data": piece, "flat_param._fqns": rel, "flat_param._shapes": [src["model"][n].shape for n in names]}
            if old_torch:
                handle["flat_param._shard_indices"] = (present[0], present[-1]) if present else (0, -1)
                handle["flat_param._shard_param_offsets"] = old_offsets
            else:
                handle["flat_param._shard_param_infos"] = tuple(infos)
            wrapped = prefix.replace("transformer.blocks.0", "transformer.blocks.0") if prefix else ""
            per_rank_model[r]["modules"].append({"name": (f"_fsdp_wrapped_module.{wrapped}" if wrapped else ""), "handles": [handle]})
    for r in range(world):
        torch.save(per_rank_model[r], folder / "model" / f"rank{r}.pt")
        torch.save(per_rank_optim[r], folder / "optim" / f"rank{r}.pt")
        torch.save({"global_step": 7}, folder / "train" / f"rank{r}.pt")


@pytest.mark.parametrize("old_torch", [False, True])
def test_local_checkpoint_unshards_to_the_full_tensors(tmp_path, old_torch):
    src = _source(1)
    folder = tmp_path / "local"
    _write_local(folder, src, world=3, old_torch=old_torch)
    assert detect_layout(folder) == "local"
    model, optim, trainer = unshard_local_checkpoint(folder)
    for n in NAMES:
        torch.testing.assert_close(model[_clean(n)], src["model"][n], rtol=0, atol=0)
        for key in ("exp_avg", "exp_avg_sq"):
            torch.testing.assert_close(optim["state"][_clean(n)][key], src["optim"]["state"][n][key], rtol=0, atol=0)
        assert float(optim["state"][_clean(n)]["step"]) == 7.0
    assert trainer["global_step"] == 7
    (folder / "model" / "rank2.pt").unlink()
    with pytest.raises(OLMoCheckpointError, match="missing shard file"):
        unshard_local_checkpoint(folder)


def test_unshard_script_reads_a_torch_legacy_directory(legacy_dir, tmp_path):
    (legacy_dir / "config.yaml").write_text((Path(__file__).resolve().parent.parent / "configs" / "tiny" / "OLMo-20M.yaml").read_text())
    out = tmp_path / "unsharded"
    proc = subprocess.run([sys.executable, str(Path(__file__).resolve().parent.parent / "scripts" / "unshard.py"), str(legacy_dir), str(out),
                           "--type", "torch_legacy"], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:]
    model = torch.load(out / "model.pt", weights_only=False)
    src = _source()
    for n in NAMES:
        torch.testing.assert_close(model[_clean(n)], src["model"][n], rtol=0, atol=0)
    assert (out / "optim.pt").is_file() and (out / "train.pt").is_file() and (out / "config.yaml").is_file()


def test_torch_new_layout_is_written_to_and_read_from_a_remote_store():
    """The distributed-checkpoint files go to a URL through the storage layer (temporary file + upload per stream) and come
    back by byte-range reads; nothing but the registered backend touches the "remote" side."""
    from pathlib import Path

    from olmo_b200 import util
    from olmo_b200.checkpoint import unshard_torch_dcp_checkpoint
    from olmo_b200.checkpoint_compat import export_torch_new_checkpoint

    class Store(util.StorageBackend):
        def __init__(self):
            self.blobs, self.range_reads = {}, 0

        def file_size(self, url):
            if url not in self.blobs:
                raise FileNotFoundError(url)
            return len(self.blobs[url])

        def get_bytes_range(self, url, start, num):
            self.range_reads += 1
            if url not in self.blobs:
                raise FileNotFoundError(url)
            return self.blobs[url][start : start + num]

        def upload(self, source, url, save_overwrite=False):
            self.blobs[url] = Path(source).read_bytes()

        def list_files(self, url):
            return sorted(k for k in self.blobs if k.startswith(url.rstrip("/") + "/"))

        def delete(self, url):
            self.blobs.pop(url, None)

    store = Store()
    util.register_storage_backend("mem", store)
    try:
        torch.manual_seed(0)
        model = {"transformer.wte.weight": torch.randn(32, 8), "transformer.blocks.0.ff_out.weight": torch.randn(8, 16)}
        optim = {
            "state": {n: {"exp_avg": torch.randn_like(t), "exp_avg_sq": torch.rand_like(t), "step": torch.tensor(7.0)} for n, t in model.items()},
            "param_groups": [{"lr": 1e-3, "params": list(model)}],
        }
        export_torch_new_checkpoint("mem://bucket/run/step7", model, optim, {"global_step": 7}, world_size=2)
        names = sorted(k[len("mem://bucket/run/step7/"):] for k in store.blobs)
        assert "model_and_optim/.metadata" in names and "train/rank1.pt" in names and any(n.endswith(".distcp") for n in names)
        assert not any(n.endswith(".tmp") for n in names)  # the metadata file was published under its final name
        got_model, got_optim, trainer = unshard_torch_dcp_checkpoint("mem://bucket/run/step7")
        assert store.range_reads > 0 and trainer == {"global_step": 7}
        for n, t in model.items():
            assert torch.equal(got_model[n], t)
            assert torch.equal(got_optim["state"][n]["exp_avg_sq"], optim["state"][n]["exp_avg_sq"])
            assert float(got_optim["state"][n]["step"]) == 7.0
        assert got_optim["param_groups"][0]["params"] == list(model)
    finally:
        util._BACKENDS.pop("mem", None)


def test_range_reader_behaves_like_a_file_under_random_seeks_and_reads():
    """Property test: the byte-range view of a remote object, wrapped in a buffered reader the way the checkpoint
    reader wraps it, returns what ``io.BytesIO`` returns for any sequence of seeks (all three origins, past either end)
    and reads (sized, to the end, zero-length)."""
    import io

    from hypothesis import given, settings
    from hypothesis import strategies as st

    from olmo_b200 import util
    from olmo_b200.checkpoint import _RangeReader

    class Store(util.StorageBackend):
        def __init__(self):
            self.blobs = {}

        def file_size(self, url):
            return len(self.blobs[url])

        def get_bytes_range(self, url, start, num):
            assert start >= 0 and num > 0 and start + num <= len(self.blobs[url])  # never asks outside the object
            return self.blobs[url][start : start + num]

    store = Store()
    util.register_storage_backend("memrr", store)
    ops = st.lists(st.one_of(
        st.tuples(st.just("seek"), st.integers(-40, 300), st.sampled_from([io.SEEK_SET, io.SEEK_CUR, io.SEEK_END])),
        st.tuples(st.just("read"), st.one_of(st.integers(0, 120), st.just(-1)), st.just(0)),
    ), min_size=1, max_size=12)

    @settings(max_examples=80, deadline=None)
    @given(size=st.integers(0, 256), buffer_size=st.sampled_from([1, 7, 64, 1024]), script=ops, seed=st.integers(0, 99))
    def check(size, buffer_size, script, seed):
        data = bytes((seed + 31 * i) % 251 for i in range(size))
        store.blobs["memrr://b/x"] = data
        ours, theirs = io.BufferedReader(_RangeReader("memrr://b/x"), buffer_size=buffer_size), io.BytesIO(data)
        for op, a, b in script:
            if op == "seek":
                if (b == io.SEEK_SET and a < 0) or (b == io.SEEK_CUR and theirs.tell() + a < 0) or (b == io.SEEK_END and size + a < 0):
                    continue  # BytesIO raises on negative absolute positions; the view clamps: not comparable
                want = theirs.seek(a, b)
                if want > size:  # BytesIO may sit past the end, the view clamps to the end: both then read nothing
                    theirs.seek(size)
                    ours.seek(a, b)
                    assert ours.read(5) == b""
                    continue
                assert ours.seek(a, b) == want
            else:
                assert ours.read(a) == theirs.read(a)
            assert ours.tell() == theirs.tell()

    try:
        check()
    finally:
        util._BACKENDS.pop("memrr", None)
