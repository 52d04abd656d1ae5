"""Data pipeline on CPU: memory-mapped token files, the deterministic iterable loader, collation."""
import numpy as np
import pytest
import torch

from olmo_b200.config import (
    CustomDatasetCollatorConfig,
    CustomDatasetConfig,
    DataConfig,
    InstanceFilterConfig,
    ModelConfig,
    PaddingDirection,
    TrainConfig,
)
from olmo_b200.data import build_collator, build_memmap_dataset, build_train_dataloader
from olmo_b200.data.collator import CustomDatasetDataCollator, DataCollator
from olmo_b200.data.custom_datasets import build_custom_dataset, extract_module_and_class
from olmo_b200.data.iterable_dataset import IterableDataset
from olmo_b200.data.memmap_dataset import MemMapDataset
from olmo_b200.data.synthetic import SyntheticTokenDataset
from olmo_b200.data.util import find_periodic_sequences, get_document_lengths


def token_file(path, values, dtype=np.uint16):
    arr = np.memmap(path, dtype=dtype, mode="w+", shape=(len(values),))
    arr[:] = values
    arr.flush()
    return path


# ------------------------------------------------------------------------------------------ memmap


def test_memmap_chunks_across_files(tmp_path):
    a = token_file(tmp_path / "a.npy", list(range(16)))
    b = token_file(tmp_path / "b.npy", list(range(16, 32 + 3)))  # trailing partial chunk is dropped
    ds = MemMapDataset(a, b, chunk_size=4, metadata=[{"label": "a"}, {"label": "b"}])
    assert len(ds) == 8 and ds.chunk_size == 4 and ds.max_seq_len == 4
    assert ds[0]["input_ids"].tolist() == [0, 1, 2, 3]
    assert ds[7]["input_ids"].tolist() == [28, 29, 30, 31]
    assert ds[-1]["input_ids"].tolist() == [28, 29, 30, 31]
    assert ds[4]["metadata"]["label"] == "b" and ds[3]["metadata"]["label"] == "a"
    assert ds[0]["input_ids"].dtype == torch.long
    with pytest.raises(IndexError):
        ds[8]


def test_memmap_label_mask_attention_mask_and_doc_lengths(tmp_path):
    ids = token_file(tmp_path / "ids.npy", [5, 6, 1, 7, 8, 9, 1, 0])
    mask = token_file(tmp_path / "mask.npy", [1, 1, 0, 1, 0, 1, 1, 0], dtype=np.bool_)
    ds = MemMapDataset(ids, chunk_size=4, label_mask_paths=[mask], generate_attention_mask=True, pad_token_id=0,
                       generate_doc_lengths=True, eos_token_id=1, include_instance_metadata=False)
    first, second = ds[0], ds[1]
    assert first["label_mask"].tolist() == [True, True, False, True]
    assert second["attention_mask"].tolist() == [1, 1, 1, 0]
    assert first["doc_lens"].tolist() == [3, 1] and second["doc_lens"].tolist() == [3, 1]
    assert "metadata" not in first
    with pytest.raises(ValueError):
        MemMapDataset(ids, chunk_size=4, generate_attention_mask=True)
    with pytest.raises(ValueError):
        MemMapDataset(ids, chunk_size=4, label_mask_paths=[mask, mask])
    with pytest.raises(ValueError):
        MemMapDataset()


def test_memmap_concat_and_instance_filter(tmp_path):
    a = MemMapDataset(token_file(tmp_path / "a.npy", list(range(8))), chunk_size=4)
    b = MemMapDataset(token_file(tmp_path / "b.npy", list(range(8, 16))), chunk_size=4)
    both = a + b
    assert len(both) == 4 and both[3]["input_ids"].tolist() == [12, 13, 14, 15]
    with pytest.raises(NotImplementedError):
        a + [1, 2, 3]

    repetitive = [7] * 40 + list(range(100, 124))
    clean = list(range(200, 264))
    ds = MemMapDataset(
        token_file(tmp_path / "r.npy", repetitive + clean), chunk_size=64,
        instance_filter_config=InstanceFilterConfig(repetition_max_period=4, repetition_min_period=1, repetition_max_count=32),
    )
    assert ds[0]["instance_mask"] is False or ds[0]["instance_mask"] == False  # noqa: E712
    assert ds[1]["instance_mask"] is True or ds[1]["instance_mask"] == True  # noqa: E712


def test_periodic_run_finder_and_document_lengths():
    arr = np.array([1, 2, 3, 9, 9, 9, 9, 9, 4, 5, 6, 4, 5, 6, 4, 5, 6, 4, 8])
    runs = {(r.start, r.end, r.period, r.times) for r in find_periodic_sequences(arr, max_period=5)}
    assert (3, 8, 1, 5) in runs
    assert (8, 18, 3, 3) in runs
    assert list(find_periodic_sequences(np.arange(50), max_period=10)) == []
    with pytest.raises(ValueError):
        list(find_periodic_sequences(np.array([1, -1, 2, 3, 4, 5]), max_period=2))
    ids = torch.tensor([3, 4, 0, 5, 0, 6, 7])
    assert get_document_lengths(ids, 0).tolist() == [3, 2, 2]
    assert get_document_lengths(torch.tensor([3, 4, 0]), 0).tolist() == [3]
    assert get_document_lengths(torch.tensor([3, 4, 5]), 0).tolist() == [3]


# --------------------------------------------------------------------------------- iterable loader


def collect(ds, n=None):
    out = []
    for item in ds:
        out.append(item["index"] if isinstance(item, dict) else item)
        if n is not None and len(out) >= n:
            break
    return out


def test_iterable_dataset_sizes_and_padding():
    data = [{"index": i} for i in range(20)]
    kw = dict(global_batch_size=4, shuffle=False)
    assert IterableDataset(data, world_size=2, rank=0, drop_last=False, **kw).total_size == 20
    assert IterableDataset(data, world_size=3, rank=0, drop_last=False, global_batch_size=3, shuffle=False).total_size == 21
    assert IterableDataset(data, world_size=3, rank=0, drop_last=True, global_batch_size=3, shuffle=False).total_size == 18
    r0 = collect(IterableDataset(data, world_size=2, rank=0, drop_last=True, **kw))
    r1 = collect(IterableDataset(data, world_size=2, rank=1, drop_last=True, **kw))
    # ranks take interleaved positions of the global order, so every global batch is split evenly
    assert r0[:4] == [0, 2, 4, 6] and r1[:4] == [1, 3, 5, 7]
    assert sorted(r0 + r1) == list(range(20))


def test_iterable_dataset_resume_and_world_size_change(tmp_path):
    data = [{"index": i} for i in range(64)]

    def order(world, start=0, seed=3, epoch=0):
        per_rank = [collect(IterableDataset(data, global_batch_size=8, seed=seed, epoch=epoch, start_index=start, world_size=world, rank=r,
                                            drop_last=True)) for r in range(world)]
        # re-assemble the global order: position k of the global stream went to rank k % world
        out = []
        for j in range(len(per_rank[0])):
            for r in range(world):
                out.append(per_rank[r][j])
        return out

    full = order(1)
    assert sorted(full) == list(range(64)) and full != list(range(64))
    assert order(2) == full and order(4) == full  # the global order does not depend on the world size
    assert order(4, start=24) == full[24:]  # resuming skips exactly the consumed examples
    assert order(1, seed=4) != full and order(1, epoch=1) != full

    ds = IterableDataset(data, global_batch_size=8, seed=3, world_size=1, rank=0, fs_local_rank=0, work_dir=tmp_path, drop_last=True)
    assert ds.global_indices_file is not None and ds.global_indices_file.is_file()
    assert collect(ds) == full
    ds.reshuffle(1)
    assert collect(ds) == order(1, epoch=1)
    capped = IterableDataset(data, global_batch_size=8, seed=3, world_size=1, rank=0, max_examples=16, drop_last=True)
    assert collect(capped) == full[:16]


class _Info:
    def __init__(self, id, num_workers):
        self.id, self.num_workers = id, num_workers


def test_iterable_dataset_splits_batches_over_workers(monkeypatch):
    data = [{"index": i} for i in range(32)]
    ds = IterableDataset(data, global_batch_size=4, shuffle=False, world_size=1, rank=0, drop_last=True)
    seen = []
    for wid in range(2):
        monkeypatch.setattr(torch.utils.data, "get_worker_info", lambda wid=wid: _Info(wid, 2))
        seen.append(collect(ds))
    # workers alternate whole device batches, so a DataLoader that round-robins them restores the order
    assert seen[0][:8] == [0, 1, 2, 3, 8, 9, 10, 11] and seen[1][:8] == [4, 5, 6, 7, 12, 13, 14, 15]
    assert sorted(seen[0] + seen[1]) == list(range(32))


# ------------------------------------------------------------------------------------------ collator


@pytest.mark.parametrize("direction", [PaddingDirection.left, PaddingDirection.right])
def test_collator_pads_every_field(direction):
    c = DataCollator(pad_direction=direction, pad_token_id=99)
    out = c([torch.tensor([1, 2, 3, 4]), torch.tensor([5, 6])])
    want = [99, 99, 5, 6] if direction == PaddingDirection.left else [5, 6, 99, 99]
    assert out["input_ids"].tolist() == [[1, 2, 3, 4], want]

    items = [
        {"input_ids": torch.tensor([1, 2, 3]), "attention_mask": torch.ones(3), "label_mask": torch.tensor([True, False, True]),
         "attention_bias": torch.zeros(3, 3), "index": 7, "instance_mask": True, "doc_lens": torch.tensor([2, 1]), "metadata": {"k": 1}},
        {"input_ids": torch.tensor([4]), "attention_mask": torch.ones(1), "label_mask": torch.tensor([True]),
         "attention_bias": torch.zeros(1, 1), "index": 8, "instance_mask": False, "doc_lens": torch.tensor([1]), "metadata": {"k": 2}},
    ]
    out = c(items)
    assert out["input_ids"].shape == (2, 3) and out["attention_mask"].shape == (2, 3) and out["label_mask"].dtype == torch.bool
    assert out["attention_bias"].shape == (2, 1, 3, 3)
    short_mask = out["attention_mask"][1].tolist()
    assert short_mask == ([0, 0, 1] if direction == PaddingDirection.left else [1, 0, 0])
    pad_pos = 0 if direction == PaddingDirection.left else 2
    assert out["attention_bias"][1, 0, pad_pos, pad_pos] == float("-inf")
    assert out["label_mask"][1].tolist() == ([False, False, True] if direction == PaddingDirection.left else [True, False, False])
    assert out["index"].tolist() == [7, 8] and out["instance_mask"].tolist() == [True, False]
    assert out["doc_lens"].tolist() == [[2, 1], [1, 0]] and out["max_doc_lens"] == [2, 1]
    assert out["metadata"] == [{"k": 1}, {"k": 2}]


def test_custom_collator_relabels_fields():
    cfg = CustomDatasetCollatorConfig(input_id_field="tokens", label_mask_field="keep")
    c = CustomDatasetDataCollator(pad_direction=PaddingDirection.right, pad_token_id=0, **{k: v for k, v in cfg.asdict().items()})
    out = c([{"tokens": [1, 2, 3], "keep": [1, 0, 1]}, {"tokens": [4], "keep": [1]}])
    assert out["input_ids"].tolist() == [[1, 2, 3], [4, 0, 0]]
    assert out["label_mask"].tolist() == [[True, False, True], [True, False, False]]


class ToyDataset(torch.utils.data.Dataset):
    def __init__(self, n: int = 5, width: int = 4):
        self.n, self.width = n, width

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        return {"input_ids": torch.full((self.width,), i)}


def toy_collate(items):
    return {"input_ids": torch.stack([x["input_ids"] for x in items]), "custom": True}


def test_custom_dataset_hooks():
    assert extract_module_and_class("pkg.mod.Cls") == ("pkg.mod", "Cls")
    assert extract_module_and_class("Cls") == (None, "Cls")
    cfg = TrainConfig(model=ModelConfig(pad_token_id=0), data=DataConfig(custom_dataset=CustomDatasetConfig(name=f"{__name__}.ToyDataset", args={"n": 3})))
    ds = build_custom_dataset(cfg)
    assert len(ds) == 3 and ds[2]["input_ids"].tolist() == [2, 2, 2, 2]
    cfg.data.custom_dataset = CustomDatasetConfig(name="ToyDataset", module=__name__, args={"n": 2}, collate_fn=f"{__name__}.toy_collate")
    assert len(build_custom_dataset(cfg)) == 2
    assert build_collator(cfg)([ToyDataset()[0]])["custom"] is True
    cfg.data.custom_dataset = CustomDatasetConfig(name="ToyDataset", module=__name__, collate_config=CustomDatasetCollatorConfig(input_id_field="input_ids"))
    assert isinstance(build_collator(cfg), CustomDatasetDataCollator)
    cfg.data.custom_dataset = None
    assert type(build_collator(cfg)) is DataCollator


# ------------------------------------------------------------------------------------------ builders


def test_builders_from_config(tmp_path):
    files = [token_file(tmp_path / f"part{i}.npy", np.arange(i * 1000, i * 1000 + 256) % 500) for i in range(2)]
    cfg = TrainConfig(
        model=ModelConfig(max_sequence_length=16, vocab_size=512, embedding_size=512, pad_token_id=0, eos_token_id=1),
        data=DataConfig(paths=[str(f) for f in files], num_workers=0, drop_last=True, pin_memory=False, prefetch_factor=None, persistent_workers=False),
        global_train_batch_size=4, device_train_batch_size=4, save_folder=str(tmp_path / "run"), save_overwrite=True,
    )
    ds = build_memmap_dataset(cfg, cfg.data)
    assert len(ds) == 32 and ds[0]["metadata"]["path"] == str(files[0])
    loader = build_train_dataloader(cfg, world_size=1, rank=0, fs_local_rank=0)
    batch = next(iter(loader))
    assert batch["input_ids"].shape == (4, 16) and "index" in batch
    assert (tmp_path / "run" / "train_data" / "global_indices.npy").is_file()

    cfg.data.paths = None
    cfg.data.datasets = {"a": [str(files[0])], "b": [str(files[1])]}
    ds = build_memmap_dataset(cfg, cfg.data)
    assert ds[0]["metadata"]["label"] == "a" and ds[31]["metadata"]["label"] == "b"
    cfg.data.datasets = None
    with pytest.raises(Exception):
        build_memmap_dataset(cfg, cfg.data)


def test_synthetic_tokens_are_reproducible():
    ds = SyntheticTokenDataset(100, 64, vocab_size=1000, eos_token_id=7, seed=5)
    a, b = ds[3]["input_ids"], SyntheticTokenDataset(100, 64, vocab_size=1000, eos_token_id=7, seed=5)[3]["input_ids"]
    assert torch.equal(a, b) and a.shape == (64,) and int(a.max()) < 1000
    assert not torch.equal(a, ds[4]["input_ids"])
    batch = ds.batch(8, 4)
    assert batch.shape == (4, 64) and torch.equal(batch[0], ds[8]["input_ids"])


def test_iterable_dataset_partition_property(monkeypatch):
    """Property test over dataset size, world size, worker count, device batch size, ``drop_last`` and restart point:
    the slices taken by all ranks and all their data-loader workers are disjoint positions of the global order and
    together cover exactly what is left of it; every rank gets the same number of instances."""
    from collections import Counter

    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=60, deadline=None)
    @given(n=st.integers(1, 90), world=st.integers(1, 5), workers=st.integers(0, 3), device_bs=st.integers(1, 4), drop_last=st.booleans(),
           consumed_batches=st.integers(0, 6), seed=st.integers(0, 99))
    def check(n, world, workers, device_bs, drop_last, consumed_batches, seed):
        data = [{"v": i} for i in range(n)]
        kw = dict(global_batch_size=device_bs * world, seed=seed, world_size=world, drop_last=drop_last, num_threads=0)
        whole = IterableDataset(data, rank=0, **kw)
        order = [int(i) for i in whole.get_global_indices()]
        assert len(order) == whole.total_size and whole.total_size % world == 0
        if drop_last:
            assert whole.total_size <= n and len(set(order)) == len(order)
        else:
            assert whole.total_size >= n and set(order) == set(range(n))  # padding repeats instances, never drops one
        start = min(consumed_batches * device_bs * world, whole.total_size)
        seen, per_rank = Counter(), []
        for rank in range(world):
            ds = IterableDataset(data, rank=rank, start_index=start, **kw)
            count = 0
            for wid in range(max(workers, 1)):
                monkeypatch.setattr(torch.utils.data, "get_worker_info", (lambda wid=wid: _Info(wid, workers)) if workers else (lambda: None))
                got = [item["index"] for item in ds]
                seen.update(got)
                count += len(got)
            per_rank.append(count)
        assert seen == Counter(order[start:])
        assert len(set(per_rank)) == 1

    check()
