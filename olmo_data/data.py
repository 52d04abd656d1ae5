"""Where package data lives (the role of the reference's ``olmo_data/data.py:9-27``): relative paths such as
``tokenizers/allenai_dolma2.json`` or ``hf_datasets/piqa/plain_text/validation`` are looked up under ``OLMO_DATA_DIR``
first, then inside this package."""
from contextlib import contextmanager
from pathlib import Path
from typing import Generator, Optional

__all__ = ["is_data_dir", "is_data_file", "get_data_path"]


def _locate(data_rel_path: str) -> Optional[Path]:
    import os

    roots = [Path(__file__).resolve().parent]
    if os.environ.get("OLMO_DATA_DIR"):
        roots.insert(0, Path(os.environ["OLMO_DATA_DIR"]))
    for root in roots:
        candidate = root / data_rel_path
        if candidate.exists():
            return candidate
    return None


def is_data_dir(data_rel_path: str) -> bool:
    found = _locate(data_rel_path)
    return found is not None and found.is_dir()


def is_data_file(data_rel_path: str) -> bool:
    found = _locate(data_rel_path)
    return found is not None and found.is_file()


@contextmanager
def get_data_path(data_rel_path: str) -> Generator[Path, None, None]:
    """Context manager yielding the on-disk path of a data file or folder (kept as a context manager so that callers
    written against a zip-safe resource API keep working)."""
    found = _locate(data_rel_path)
    if found is None:
        raise FileNotFoundError(f"'{data_rel_path}' is neither under OLMO_DATA_DIR nor inside the olmo_data package")
    yield found
