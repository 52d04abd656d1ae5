"""The host-side token reader: extent table, batched reads through the C++ reader and through byte-range reads."""
import pickle

import numpy as np
import pytest
import torch

from olmo_b200.data import MemMapDataset
from olmo_b200.data import token_store as ts


def _files(tmp_path, dtype, lengths, seed=0):
    rng = np.random.default_rng(seed)
    paths, arrays = [], []
    for i, n in enumerate(lengths):
        arr = rng.integers(0, np.iinfo(dtype).max, size=n, dtype=dtype)
        path = tmp_path / f"part{i}.npy"
        arr.tofile(path)
        paths.append(str(path))
        arrays.append(arr)
    return paths, arrays


def _expected(arrays, chunk):
    rows = [a[: len(a) // chunk * chunk].reshape(-1, chunk) for a in arrays]
    return np.concatenate(rows).astype(np.int64)


@pytest.mark.parametrize("dtype", [np.uint8, np.uint16, np.uint32, np.uint64])
def test_native_and_fallback_reads_agree_with_numpy(tmp_path, dtype, monkeypatch):
    chunk = 16
    paths, arrays = _files(tmp_path, dtype, [5 * chunk + 3, 7, 2 * chunk, chunk - 1, 3 * chunk + 15])  # two files hold no whole chunk
    want = _expected(arrays, chunk)
    if dtype == np.uint64:
        want = np.concatenate([a[: len(a) // chunk * chunk].reshape(-1, chunk) for a in arrays]).view(np.int64)
    store = ts.TokenStore(paths, dtype, chunk, threads=3)
    assert len(store) == 10 and store.file_ranges() == [(0, 5), (5, 5), (5, 7), (7, 7), (7, 10)]
    files, chunks = store.locate([0, 4, 5, 6, 7, 9, -1])
    assert files.tolist() == [0, 0, 2, 2, 4, 4, 4] and chunks.tolist() == [0, 4, 0, 1, 0, 2, 2]
    order = [9, 0, 5, 5, 3, -3]
    assert ts.native_reader_available(), "g++ is part of the build environment: the C++ reader must load"
    native = store.read(order)
    assert torch.equal(native, torch.from_numpy(want[[9, 0, 5, 5, 3, 7]]))
    monkeypatch.setattr(ts.TokenStore, "_native", lambda self: None)
    assert torch.equal(ts.TokenStore(paths, dtype, chunk).read(order), native)
    with pytest.raises(IndexError):
        store.locate([10])
    assert store.read([]).shape == (0, chunk)
    clone = pickle.loads(pickle.dumps(store))  # what a data-loader worker receives
    assert clone._handle is None and torch.equal(clone.read([2]), native.new_tensor(want[[2]]))


def test_reader_reports_a_file_that_shrank(tmp_path):
    paths, arrays = _files(tmp_path, np.uint16, [64, 64])
    store = ts.TokenStore(paths, np.uint16, 16)
    assert len(store) == 8
    arrays[1][:20].tofile(paths[1])  # truncated after the extent table was built
    with pytest.raises(OSError, match="part1"):
        store.read([7])
    out = torch.empty(1, 16, dtype=torch.int64)
    assert store.read([4], out=out) is out and out[0].tolist() == arrays[1][:16].astype(np.int64).tolist()


def test_dataset_batches_match_single_items(tmp_path):
    chunk = 8
    paths, arrays = _files(tmp_path, np.uint16, [3 * chunk, 5, 2 * chunk + 1])
    masks = []
    for i, a in enumerate(arrays):
        m = (np.arange(len(a)) % 3 == 0)
        path = tmp_path / f"mask{i}.npy"
        m.astype(np.bool_).tofile(path)
        masks.append(str(path))
    eos = int(arrays[0][3])
    ds = MemMapDataset(*paths, chunk_size=chunk, metadata=[{"f": 0}, {"f": 1}, {"f": 2}], label_mask_paths=masks, generate_attention_mask=True,
                       pad_token_id=int(arrays[2][1]), generate_doc_lengths=True, eos_token_id=eos)
    assert len(ds) == 5 and ds.offsets == [(0, 3), (3, 3), (3, 5)]
    items = ds.__getitems__([4, 0, 3])
    for got, idx in zip(items, [4, 0, 3]):
        one = ds[idx]
        assert set(got) == set(one) == {"input_ids", "label_mask", "metadata", "attention_mask", "doc_lens"}
        for key in ("input_ids", "label_mask", "attention_mask", "doc_lens"):
            assert torch.equal(got[key], one[key]), key
        assert got["metadata"] == one["metadata"]
    assert items[0]["metadata"] == {"f": 2} and items[2]["attention_mask"][1] == 0 and items[1]["label_mask"].tolist() == [True, False, False] * 2 + [True, False]
    assert int(items[1]["doc_lens"].sum()) == chunk and items[1]["doc_lens"][0] == 4  # first document ends at the end-of-text token
    batch = ds.read_batch([1, 2])
    assert batch["input_ids"].shape == (2, chunk) and batch["label_mask"].dtype == torch.bool
    loader = torch.utils.data.DataLoader(ds, batch_size=2, collate_fn=lambda rows: torch.stack([r["input_ids"] for r in rows]))
    assert torch.equal(torch.cat(list(loader)), torch.from_numpy(_expected(arrays, chunk)))
    # a mask file of the wrong length is refused
    np.zeros(7, dtype=np.bool_).tofile(masks[0])
    with pytest.raises(ValueError, match="same size"):
        len(MemMapDataset(*paths, chunk_size=chunk, label_mask_paths=masks))


def test_locate_and_read_against_brute_force_on_random_layouts(tmp_path):
    """Property test: for random file lengths (files shorter than a chunk and empty files included), chunk sizes and
    index sets, ``locate`` agrees with walking the files one by one, and ``read`` returns exactly the tokens numpy sees."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    counter = [0]

    @settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
    @given(lengths=st.lists(st.integers(0, 70), min_size=1, max_size=6), chunk=st.integers(1, 9), seed=st.integers(0, 2**16))
    def check(lengths, chunk, seed):
        counter[0] += 1
        folder = tmp_path / f"case{counter[0]}"
        folder.mkdir()
        rng = np.random.default_rng(seed)
        paths, arrays = [], []
        for i, n in enumerate(lengths):
            arr = rng.integers(0, 60000, size=n, dtype=np.uint16)
            arr.tofile(folder / f"f{i}.npy")
            paths.append(str(folder / f"f{i}.npy"))
            arrays.append(arr)
        store = ts.TokenStore(paths, np.uint16, chunk, threads=3)
        expected = [(f, c) for f, arr in enumerate(arrays) for c in range(len(arr) // chunk)]
        assert len(store) == len(expected)
        assert store.chunks_per_file().tolist() == [len(a) // chunk for a in arrays]
        if not expected:
            assert store.read([]).shape == (0, chunk)
            with pytest.raises(IndexError):
                store.locate([0])
            return
        picks = rng.integers(-len(expected), len(expected), size=min(12, 2 * len(expected)))
        files, chunks = store.locate(picks)
        assert [(int(f), int(c)) for f, c in zip(files, chunks)] == [expected[int(i)] for i in picks]
        got = store.read(picks)
        want = np.stack([arrays[f][c * chunk:(c + 1) * chunk].astype(np.int64) for f, c in (expected[int(i)] for i in picks)])
        assert got.dtype == torch.int64 and np.array_equal(got.numpy(), want)
        with pytest.raises(IndexError):
            store.locate([len(expected)])
        store.close()

    check()
