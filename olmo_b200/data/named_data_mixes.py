"""
Named data mixes: a mix name maps to an ordered list of token-file paths relative to a storage root.

The reference hard-codes three mixes as a 3,000-line literal (``olmo/data/named_data_mixes.py``); the lists name files in
AI2's buckets and are data, not code.  Here a mix is a text file with one relative path per line (``#`` comments and
blank lines ignored), looked up as ``data_mixes/<name>.txt`` in every packaged-data root (``OLMO_DATA_DIR`` first) or
registered at run time with :func:`register_mix`.  ``DATA_PATHS`` keeps the reference's mapping interface.
"""
from __future__ import annotations

from pathlib import Path
from typing import Dict, Iterator, List, Mapping, Sequence

__all__ = ["DATA_PATHS", "register_mix", "load_mix_file", "resolve_mix"]

_REGISTERED: Dict[str, List[str]] = {}


def load_mix_file(path) -> List[str]:
    lines = []
    for line in Path(path).read_text().splitlines():
        line = line.split("#", 1)[0].strip()
        if line:
            lines.append(line)
    return lines


def register_mix(name: str, paths: Sequence[str]) -> None:
    _REGISTERED[name] = list(paths)


class _Mixes(Mapping):
    def _on_disk(self) -> Dict[str, Path]:
        from ..util import _data_roots

        found: Dict[str, Path] = {}
        for root in _data_roots():
            folder = Path(root) / "data_mixes"
            if folder.is_dir():
                for f in sorted(folder.glob("*.txt")):
                    found.setdefault(f.stem, f)
        return found

    def __getitem__(self, name: str) -> List[str]:
        if name in _REGISTERED:
            return list(_REGISTERED[name])
        files = self._on_disk()
        if name in files:
            return load_mix_file(files[name])
        if Path(name).is_file():
            return load_mix_file(name)
        raise KeyError(f"unknown data mix '{name}': put data_mixes/{name}.txt under OLMO_DATA_DIR, pass a file path, or call register_mix()")

    def __iter__(self) -> Iterator[str]:
        return iter(sorted(set(_REGISTERED) | set(self._on_disk())))

    def __len__(self) -> int:
        return len(set(_REGISTERED) | set(self._on_disk()))


DATA_PATHS: Mapping = _Mixes()


def resolve_mix(name: str, read_location: str) -> List[str]:
    """Absolute paths/URLs of a mix under ``read_location``."""
    root = read_location.rstrip("/")
    return [f"{root}/{p}" for p in DATA_PATHS[name]]
