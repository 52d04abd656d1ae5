"""Utilities: storage back ends (with an in-memory fake for a remote scheme), checkpoint discovery, resource caching,
generators, dictionary helpers, the safetensors flavour, torch helpers."""
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from olmo_b200 import util
from olmo_b200.exceptions import OLMoThreadError
from olmo_b200.safetensors_util import safetensors_file_to_state_dict, state_dict_to_safetensors_file
from olmo_b200.torch_util import ensure_finite_, get_cumulative_document_lengths, move_to_device, seed_all


class MemoryBackend(util.StorageBackend):
    """A remote store held in a dictionary: exercises every code path that goes through the scheme registry."""

    def __init__(self):
        self.blobs = {}
        self.reads = 0

    def file_size(self, url):
        if url not in self.blobs:
            raise FileNotFoundError(url)
        return len(self.blobs[url])

    def get_bytes_range(self, url, start, num):
        self.reads += 1
        if url not in self.blobs:
            raise FileNotFoundError(url)
        return self.blobs[url][start : start + num]

    def upload(self, source, url, save_overwrite=False):
        if url in self.blobs and not save_overwrite:
            raise FileExistsError(url)
        self.blobs[url] = Path(source).read_bytes()

    def list_files(self, url):
        prefix = url.rstrip("/") + "/"
        return sorted(k for k in self.blobs if k.startswith(prefix))

    def delete(self, url):
        self.blobs.pop(url, None)

    def find_latest_checkpoint(self, url):
        names = {k[len(url.rstrip("/")) + 1 :].split("/")[0] for k in self.list_files(url)}
        best = util._pick_latest(n for n in names if n.startswith("step"))
        return None if best is None else f"{url.rstrip('/')}/{best}"


@pytest.fixture()
def mem():
    backend = MemoryBackend()
    util.register_storage_backend("mem", backend)
    yield backend
    util._BACKENDS.pop("mem", None)


def test_remote_scheme_round_trip(mem, tmp_path, monkeypatch):
    src = tmp_path / "blob.bin"
    src.write_bytes(bytes(range(200)))
    util.upload(src, "mem://bucket/run/step10/blob.bin")
    assert util.file_size("mem://bucket/run/step10/blob.bin") == 200
    assert util.get_bytes_range("mem://bucket/run/step10/blob.bin", 10, 5) == bytes(range(10, 15))
    with pytest.raises(FileExistsError):
        util.upload(src, "mem://bucket/run/step10/blob.bin")
    util.upload(src, "mem://bucket/run/step10/blob.bin", save_overwrite=True)
    util.upload(src, "mem://bucket/run/step200-unsharded/blob.bin")
    assert util.list_files("mem://bucket/run") == ["mem://bucket/run/step10/blob.bin", "mem://bucket/run/step200-unsharded/blob.bin"]
    assert util.find_latest_checkpoint("mem://bucket/run") == "mem://bucket/run/step200-unsharded"
    with pytest.raises(FileNotFoundError):
        util.file_size("mem://bucket/missing")

    # remote files are fetched once into the cache directory
    monkeypatch.setenv("OLMO_CACHE_DIR", str(tmp_path / "cache"))
    first = util.resource_path("mem://bucket/run/step10", "blob.bin")
    reads = mem.reads
    second = util.resource_path("mem://bucket/run/step10", "blob.bin")
    assert first == second and first.read_bytes() == bytes(range(200)) and mem.reads == reads
    util.delete_file("mem://bucket/run/step10/blob.bin")
    assert util.list_files("mem://bucket/run") == ["mem://bucket/run/step200-unsharded/blob.bin"]
    with pytest.raises(Exception):
        util.file_size("nosuchscheme://x/y")


def test_token_files_stream_from_a_remote_scheme(mem, tmp_path):
    from olmo_b200.data import MemMapDataset

    arr = np.arange(64, dtype=np.uint16)
    f = tmp_path / "tokens.npy"
    arr.tofile(f)
    util.upload(f, "mem://bucket/data/tokens.npy")
    ds = MemMapDataset("mem://bucket/data/tokens.npy", chunk_size=16)
    assert len(ds) == 4 and ds[2]["input_ids"].tolist() == list(range(32, 48))


def test_local_checkpoint_discovery_and_small_helpers(tmp_path):
    assert util.find_latest_checkpoint(tmp_path) is None
    for name in ("step5", "step100", "step100-unsharded", "step20-unsharded", "notes"):
        (tmp_path / name).mkdir()
    assert Path(util.find_latest_checkpoint(tmp_path)).name == "step100"  # sharded wins a tie
    (tmp_path / "step300-unsharded").mkdir()
    assert Path(util.find_latest_checkpoint(tmp_path)).name == "step300-unsharded"
    empty = tmp_path / "empty"
    assert util.dir_is_empty(empty)
    empty.mkdir()
    assert util.dir_is_empty(empty)
    (empty / "x").write_text("1")
    assert not util.dir_is_empty(empty)
    assert util.clean_opt("--model.d_model=4") == "model.d_model=4" and util.clean_opt("-x=1") == "x=1" and util.clean_opt("--flag") == "flag=True"
    assert util.is_url("s3://a/b") and util.is_url("https://x") and not util.is_url("/tmp/x") and not util.is_url("relative/path")
    assert util.flatten_dict({"a": {"b": 1, "c": {"d": 2}}, "e": [1, 2]}) == {"a.b": 1, "a.c.d": 2, "e": [1, 2]}
    assert util.flatten_dict({"e": [1, {"f": 3}]}, include_lists=True) == {"e.0": 1, "e.1.f": 3}
    util.wait_for(lambda: True, "instant")
    with pytest.raises(TimeoutError):
        util.wait_for(lambda: False, "never", timeout=0.2)


def test_generators():
    assert list(util.roundrobin("ABC", "D", "EF")) == list("ADEBFC")
    assert list(util.threaded_generator(iter(range(100)), maxsize=4)) == list(range(100))

    def broken():
        yield 1
        raise ValueError("boom")

    with pytest.raises(OLMoThreadError):
        list(util.threaded_generator(broken(), thread_name="t"))


def test_safetensors_flavour_round_trip(tmp_path):
    state = {
        "model": {"w": torch.randn(3, 4), "nested": {"b": torch.arange(5)}},
        "step": 7,
        "names": ["a", "b"],
        "bf16": torch.randn(2, 2).to(torch.bfloat16),
        ("tuple", "key"): torch.ones(1),
    }
    path = tmp_path / "state.safetensors"
    state_dict_to_safetensors_file(state, path)
    back = safetensors_file_to_state_dict(path)
    assert back["step"] == 7 and back["names"] == ["a", "b"]
    torch.testing.assert_close(back["model"]["w"], state["model"]["w"])
    assert torch.equal(back["model"]["nested"]["b"], state["model"]["nested"]["b"])
    assert back["bf16"].dtype == torch.bfloat16 and torch.equal(back[("tuple", "key")], torch.ones(1))


def test_torch_helpers():
    dl = torch.tensor([[3, 5, 0], [2, 2, 4]])
    assert get_cumulative_document_lengths(dl).tolist() == [0, 3, 8, 10, 12, 16]
    moved = move_to_device({"a": torch.ones(2), "b": [torch.zeros(1), 3], "c": "text"}, torch.device("cpu"))
    assert moved["c"] == "text" and moved["b"][1] == 3 and moved["a"].device.type == "cpu"
    x = torch.tensor([float("-inf"), 1.0, float("inf")])
    ensure_finite_(x, check_neg_inf=True, check_pos_inf=True)
    assert torch.isfinite(x).all() and x[0] == torch.finfo(torch.float32).min and x[2] == torch.finfo(torch.float32).max
    seed_all(3)
    a = torch.rand(3)
    seed_all(3)
    assert torch.equal(a, torch.rand(3))
    with pytest.raises(ValueError):
        seed_all(-1)


def test_rank_helpers_read_the_launcher_environment(monkeypatch):
    from olmo_b200 import torch_util as T

    for k, v in {"RANK": "5", "WORLD_SIZE": "16", "LOCAL_RANK": "1", "LOCAL_WORLD_SIZE": "4", "NODE_RANK": "1"}.items():
        monkeypatch.setenv(k, v)
    assert T.get_global_rank() == 5 and T.get_local_rank() == 1 and T.get_local_world_size() == 4
    assert T.get_world_size() == 1  # the world size comes from the process group, which this test never creates
    assert T.get_node_rank() == 1
    monkeypatch.delenv("OLMO_SHARED_FS", raising=False)
    monkeypatch.delenv("FS_LOCAL_RANK", raising=False)
    assert T.get_fs_local_rank() == 1  # node-local file system: the local rank decides who writes
    monkeypatch.setenv("OLMO_SHARED_FS", "1")
    assert T.get_fs_local_rank() == 5  # shared file system: only global rank 0 writes
    monkeypatch.setenv("FS_LOCAL_RANK", "0")
    assert T.get_fs_local_rank() == 0


def test_olmo_data_package_locates_files(tmp_path, monkeypatch):
    from olmo_data.data import get_data_path, is_data_dir, is_data_file

    assert is_data_dir("tokenizers") and not is_data_file("tokenizers/absent.json")
    (tmp_path / "tokenizers").mkdir()
    (tmp_path / "tokenizers" / "mine.json").write_text("{}")
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))
    assert is_data_file("tokenizers/mine.json")
    with get_data_path("tokenizers/mine.json") as path:
        assert path == tmp_path / "tokenizers" / "mine.json"
    with pytest.raises(FileNotFoundError):
        with get_data_path("hf_datasets/none"):
            pass


def test_dataset_saver_writes_where_the_loader_looks_and_hooks_are_public(tmp_path, monkeypatch, capsys):
    datasets = pytest.importorskip("datasets")
    from olmo_b200.exceptions import OLMoCliError

    ds = datasets.Dataset.from_dict({"question": ["a", "b"], "label": [0, 1]})
    folder = util.save_hf_dataset_to_disk(ds, "toy/set", None, "validation", tmp_path / "hf_datasets")
    assert folder == tmp_path / "hf_datasets" / "toy" / "set" / "none" / "validation"
    monkeypatch.setenv("OLMO_DATA_DIR", str(tmp_path))
    assert list(util.load_hf_dataset("toy/set", None, "validation")["question"]) == ["a", "b"]
    util.excepthook(OLMoCliError, OLMoCliError("bad flag"), None)
    assert "bad flag" in capsys.readouterr().err
    bar = util.get_progress_bar()
    task = bar.add_task("fetch", total=10)
    bar.update(task, advance=10)
    assert bar.tasks[0].finished


def test_rich_handler_formats_records_and_tracebacks():
    rich = pytest.importorskip("rich")
    import io
    import logging

    from rich.console import Console

    previous = rich.get_console()
    buffer = io.StringIO()
    rich._console = Console(file=buffer, width=200, force_terminal=False)
    logger = logging.getLogger("rich-handler-test")
    handler = util.RichHandler()
    logger.addHandler(handler)
    logger.setLevel(logging.INFO)
    logger.propagate = False
    try:
        logger.info("hello %s", "world")  # (the rank shown comes from the record factory that setup_logging installs, when it ran)
        try:
            raise ValueError("boom")
        except ValueError:
            logger.exception("failed")
    finally:
        logger.removeHandler(handler)
        rich._console = previous
    out = buffer.getvalue()
    assert "hello world" in out and "rank=" in out and "[rich-handler-test:" in out and "ValueError" in out and "boom" in out


def test_safetensors_flavour_round_trips_random_nested_states(tmp_path):
    """Property test: nested dictionaries of tensors (several dtypes, zero-size, non-contiguous, views of one buffer) and
    plain Python leaves (numbers, strings, ``None``, lists, empty dictionaries) come back equal, types included."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    dtypes = [torch.float32, torch.bfloat16, torch.int64, torch.uint8, torch.bool, torch.float16]
    flat = torch.arange(64, dtype=torch.float32)

    def tensor_of(kind, seed):
        g = torch.Generator().manual_seed(seed)
        if kind == "view":
            a = seed % 32
            return flat[a : a + 8 + seed % 8]
        if kind == "transposed":
            return torch.randn(3, 4, generator=g).t()
        if kind == "empty":
            return torch.zeros(0, 5)
        if kind == "scalar":
            return torch.tensor(float(seed))
        return (torch.randn(2, 3, generator=g) * 5).to(dtypes[seed % len(dtypes)])

    tensors = st.builds(tensor_of, st.sampled_from(["view", "transposed", "empty", "scalar", "dense"]), st.integers(0, 1000))
    plain = st.one_of(st.integers(-5, 5), st.floats(-1, 1), st.text(max_size=5), st.none(), st.lists(st.integers(0, 3), max_size=3), st.just({}))
    keys = st.one_of(st.text(alphabet="abc._", min_size=1, max_size=6), st.integers(0, 9))
    trees = st.recursive(st.one_of(tensors, plain), lambda kids: st.dictionaries(keys, kids, min_size=1, max_size=4), max_leaves=10)

    def same(a, b):
        if isinstance(a, torch.Tensor):
            return isinstance(b, torch.Tensor) and a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)
        if isinstance(a, dict):
            return isinstance(b, dict) and a.keys() == b.keys() and all(same(a[k], b[k]) for k in a)
        return type(a) is type(b) and a == b

    @settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture, HealthCheck.too_slow])
    @given(st.dictionaries(keys, trees, min_size=0, max_size=4))
    def check(state):
        path = tmp_path / "s.safetensors"
        state_dict_to_safetensors_file(state, path)
        assert same(state, safetensors_file_to_state_dict(path))

    check()
