"""Builders that turn the data sections of a training config into datasets, collators and loaders
(the public functions of the reference's ``olmo/data/__init__.py:22-180``)."""
from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple, cast

from torch.utils.data import DataLoader, DistributedSampler

from ..aliases import PathOrStr
from ..config import DataConfig, TrainConfig
from ..exceptions import OLMoConfigurationError
from ..torch_util import barrier, get_global_rank, get_world_size
from .collator import CustomDatasetDataCollator, DataCollator
from .custom_datasets import build_custom_collate_fn, build_custom_dataset, extract_module_and_class
from .iterable_dataset import IterableDataset
from .memmap_dataset import MemMapDataset
from .synthetic import SyntheticTokenDataset

__all__ = [
    "MemMapDataset", "DataCollator", "IterableDataset", "SyntheticTokenDataset", "build_eval_dataloader",
    "build_train_dataloader", "build_memmap_dataset", "build_collator", "build_custom_dataset", "extract_module_and_class",
]


def _token_sources(data_config: DataConfig) -> Tuple[List[str], List[Dict[str, Any]]]:
    """Token files of a data section with one metadata record per file: either a flat ``paths`` list (record: the path)
    or labelled groups in ``datasets`` (record: the label; groups in label order)."""
    if data_config.paths and data_config.datasets:
        raise OLMoConfigurationError("DataConfig.paths is mutually exclusive with DataConfig.datasets")
    if data_config.paths:
        return list(data_config.paths), [{"path": str(p)} for p in data_config.paths]
    if data_config.datasets:
        labelled = [(label, path) for label in sorted(data_config.datasets) for path in data_config.datasets[label]]
        return [path for _, path in labelled], [{"label": label} for label, _ in labelled]
    raise OLMoConfigurationError("One of DataConfig.paths or DataConfig.datasets is required")


def _loader_options(data_config: DataConfig) -> Dict[str, Any]:
    """``DataLoader`` keywords that depend only on the data section (worker options are void without workers)."""
    workers = data_config.num_workers
    return {
        "num_workers": workers, "pin_memory": data_config.pin_memory, "timeout": data_config.timeout,
        "prefetch_factor": data_config.prefetch_factor if workers else None,
        "persistent_workers": bool(workers) and data_config.persistent_workers,
    }


def _data_seed(train_config: TrainConfig, data_config: DataConfig) -> int:
    return train_config.seed if data_config.seed is None else data_config.seed


def build_memmap_dataset(train_config: TrainConfig, data_config: DataConfig, include_instance_metadata: bool = True) -> MemMapDataset:
    """The token dataset of one data section (reference: ``olmo/data/__init__.py:22-53``)."""
    paths, metadata = _token_sources(data_config)
    model = train_config.model
    return MemMapDataset(
        *paths, chunk_size=model.max_sequence_length, memmap_dtype=data_config.effective_memmap_dtype, metadata=metadata,
        include_instance_metadata=include_instance_metadata, pad_token_id=model.pad_token_id, eos_token_id=model.eos_token_id,
        generate_attention_mask=data_config.generate_attention_mask, generate_doc_lengths=data_config.generate_doc_lengths,
        label_mask_paths=cast(Optional[List[PathOrStr]], data_config.label_mask_paths), instance_filter_config=data_config.instance_filter,
    )


#: collator keyword -> attribute of ``custom_dataset.collate_config`` naming the item field it reads
_COLLATE_FIELDS = ("input_id", "attention_mask", "attention_bias", "label_mask", "index", "instance_mask", "doc_lens", "metadata")


def build_collator(train_config: TrainConfig) -> DataCollator:
    """Default collator, a collator reading user-named fields, or a user-supplied callable (``olmo/data/__init__.py:56-89``)."""
    custom = train_config.data.custom_dataset
    if custom is None:
        return DataCollator.from_train_config(train_config)
    if custom.collate_fn:
        try:
            return build_custom_collate_fn(train_config)  # type: ignore[return-value]
        except AttributeError:
            raise OLMoConfigurationError(
                f"collate_fn {custom.collate_fn} not found. Please specify the full module path of the function."
            ) from None
    fields = custom.collate_config
    renames = {} if fields is None else {f"{name}_field": getattr(fields, f"{name}_field") for name in _COLLATE_FIELDS}
    return CustomDatasetDataCollator(pad_direction=train_config.data.pad_direction, pad_token_id=train_config.model.pad_token_id, **renames)


def build_eval_dataloader(train_config: TrainConfig, data_config: DataConfig, batch_size: int, shuffle: bool = True) -> DataLoader:
    """Evaluation loader: every rank gets its stride of the (optionally shuffled) dataset (``olmo/data/__init__.py:92-125``)."""
    dataset = build_memmap_dataset(train_config, data_config, include_instance_metadata=True)
    world = get_world_size()
    if data_config.drop_last:
        batch_size = min(batch_size, len(dataset) // world)  # at least one full batch per rank, or none at all
        assert batch_size > 0, f"dataset for {data_config.paths} is too small"
    sampler = DistributedSampler(dataset, drop_last=data_config.drop_last, shuffle=shuffle, num_replicas=world, rank=get_global_rank(),
                                 seed=_data_seed(train_config, data_config))
    collator = DataCollator(pad_direction=data_config.pad_direction, pad_token_id=train_config.model.pad_token_id)
    return DataLoader(dataset, batch_size=batch_size, collate_fn=collator, sampler=sampler, **_loader_options(data_config))


def _train_work_dir(train_config: TrainConfig) -> Path:
    """``save_folder/train_data`` holds the persisted global order; an existing one is only reused with ``save_overwrite``."""
    work_dir = Path(train_config.save_folder) / "train_data"
    if get_global_rank() == 0:
        if work_dir.is_dir() and not train_config.save_overwrite:
            raise OLMoConfigurationError("train data working directory already exists, use --save_overwrite to overwrite")
        work_dir.mkdir(exist_ok=True, parents=True)
    barrier()
    return work_dir


def build_train_dataloader(
    train_config: TrainConfig, *, world_size: Optional[int] = None, rank: Optional[int] = None,
    fs_local_rank: Optional[int] = None, include_instance_metadata: bool = False,
) -> DataLoader:
    """Training loader over the deterministic, restartable global order (``olmo/data/__init__.py:128-180``)."""
    assert train_config.device_train_batch_size is not None
    data = train_config.data
    collator = build_collator(train_config)
    if data.custom_dataset:
        if data.paths is not None or data.datasets is not None:
            raise OLMoConfigurationError("custom_dataset_class is mutually exclusive with DataConfig.paths and DataConfig.datasets")
        dataset = build_custom_dataset(train_config)
        collator = build_custom_collate_fn(train_config) or collator  # type: ignore[assignment]
    else:
        dataset = build_memmap_dataset(train_config, data, include_instance_metadata=include_instance_metadata)
    ordered = IterableDataset(
        dataset,  # type: ignore[arg-type]
        train_config.global_train_batch_size, seed=_data_seed(train_config, data), epoch=train_config.epoch or 0, shuffle=True,
        drop_last=data.drop_last, world_size=world_size, rank=rank, fs_local_rank=fs_local_rank, work_dir=_train_work_dir(train_config),
    )
    return DataLoader(ordered, batch_size=train_config.device_train_batch_size, drop_last=data.drop_last, collate_fn=collator,
                      **_loader_options(data))
