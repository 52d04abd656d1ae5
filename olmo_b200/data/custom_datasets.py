"""Import-by-name plumbing for user-supplied datasets (reference: ``olmo/data/custom_datasets.py:15-55``)."""
from __future__ import annotations

from importlib import import_module
from typing import Any, Callable, Optional

from torch.utils.data import Dataset

from ..config import TrainConfig
from ..exceptions import OLMoConfigurationError

__all__ = ["build_custom_dataset", "extract_module_and_class"]


def extract_module_and_class(name: str):
    """``"pkg.mod.Cls"`` -> ``("pkg.mod", "Cls")``; a bare name has module ``None``."""
    if "." in name:
        module, _, cls = name.rpartition(".")
        return module, cls
    return None, name


def _resolve(name: str, module: Optional[str]) -> Callable[..., Any]:
    mod, attr = extract_module_and_class(name)
    mod = mod or module
    if mod is None:
        raise OLMoConfigurationError(f"cannot tell which module defines '{name}'; set custom_dataset.module")
    return getattr(import_module(mod), attr)


def build_custom_dataset(train_config: TrainConfig) -> Dataset:
    custom = train_config.data.custom_dataset
    assert custom is not None
    factory = _resolve(custom.name, custom.module)
    return factory(**(custom.args or {}))


def build_custom_collate_fn(train_config: TrainConfig) -> Optional[Callable]:
    custom = train_config.data.custom_dataset
    assert custom is not None
    if custom.collate_fn is None:
        return None
    module = custom.module or extract_module_and_class(custom.name)[0]
    return _resolve(custom.collate_fn, module)
