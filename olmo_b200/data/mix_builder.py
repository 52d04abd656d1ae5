"""
Assemble the token-file list of a training (anneal, micro-anneal) run from *sources*.

A source is a folder or URL prefix holding token files (``.npy`` memmaps) plus how much of it to take: everything, a
fraction, an absolute token count, or a repetition factor above one.  Files are taken whole, in a seeded random order,
until the source's target is reached — the procedure of the reference's ``scripts/peteish7_config_maker.py`` and
``scripts/microanneal_config_maker.py`` (``get_token_strs``), here on top of the framework's storage layer (local paths,
``s3://``, ``r2://``, ``gs://``, ``weka://``), reproducible from a seed, and returning data instead of appending text to a
YAML template.  ``examine`` gives the per-source token table of any path list (the reference's ``examine_config``).
"""
from __future__ import annotations

import random
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence, Tuple, Union

from ..util import file_size, is_url, list_files

__all__ = ["Source", "list_token_files", "select_files", "build_mix", "examine", "human_count", "parse_source"]


@dataclass
class Source:
    """Where token files are and how much of them a mix takes (at most one of ``fraction`` / ``tokens`` / ``repeat``)."""

    prefix: str
    fraction: Optional[float] = None  # share of the source's tokens, 0 < f <= 1
    tokens: Optional[float] = None  # absolute target
    repeat: Optional[float] = None  # > 1: the whole source this many times (whole passes, then a partial one)
    name: Optional[str] = None
    files: List[Tuple[str, int]] = field(default_factory=list, repr=False)  # filled by list_token_files()

    def __post_init__(self) -> None:
        given = [x for x in (self.fraction, self.tokens, self.repeat) if x is not None]
        if len(given) > 1:
            raise ValueError(f"source {self.prefix}: give at most one of fraction, tokens, repeat")
        if self.fraction is not None and not 0 < self.fraction <= 1:
            raise ValueError(f"source {self.prefix}: fraction must be in (0, 1]; use repeat for more than one pass")
        if self.repeat is not None and self.repeat < 1:
            raise ValueError(f"source {self.prefix}: repeat must be at least 1; use fraction for less than one pass")


def parse_source(text: str) -> Source:
    """``PREFIX``, ``PREFIX=0.25`` (fraction), ``PREFIX=3e9`` or ``PREFIX=3B`` (tokens), ``PREFIX=x2`` (repeat)."""
    prefix, sep, amount = text.rpartition("=")
    if not sep or "://" in amount or "/" in amount:
        return Source(text)
    amount = amount.strip()
    if amount.lower().startswith("x"):
        return Source(prefix, repeat=float(amount[1:]))
    scale = {"k": 1e3, "m": 1e6, "b": 1e9, "g": 1e9, "t": 1e12}.get(amount[-1].lower())
    value = float(amount[:-1]) * scale if scale else float(amount)
    return Source(prefix, fraction=value) if value <= 1 and scale is None else Source(prefix, tokens=value)


def list_token_files(prefix: str, extension: str = ".npy", threads: int = 16) -> List[Tuple[str, int]]:
    """``(path or URL, size in bytes)`` of every ``*extension`` file below ``prefix``, sorted by name."""
    if is_url(prefix):
        found = [u for u in list_files(prefix) if u.endswith(extension)]
    else:
        root = Path(prefix)
        found = sorted(str(p) for p in (root.rglob(f"*{extension}") if root.is_dir() else [])) or ([prefix] if root.is_file() else [])
    if not found:
        raise FileNotFoundError(f"no *{extension} files under {prefix}")
    with ThreadPoolExecutor(max_workers=threads) as pool:
        sizes = list(pool.map(file_size, found))
    return sorted(zip(found, sizes))


def select_files(files: Sequence[Tuple[str, int]], target_tokens: float, bytes_per_token: int, rng: random.Random) -> List[Tuple[str, int]]:
    """Whole files in a random order until at least ``target_tokens`` are covered (all of them if they hold less)."""
    order = list(files)
    rng.shuffle(order)
    taken, covered = [], 0
    for path, size in order:
        if covered >= target_tokens:
            break
        taken.append((path, size))
        covered += size // bytes_per_token
    return taken


def build_mix(sources: Iterable[Union[Source, str]], *, bytes_per_token: int = 4, seed: int = 0, extension: str = ".npy"
              ) -> Tuple[List[str], List[Dict[str, object]]]:
    """The ordered path list of a mix and one table row per source (``source``, ``files``, ``tokens``, ``available``,
    ``share``).  The same seed and the same listings give the same mix."""
    paths: List[str] = []
    rows: List[Dict[str, object]] = []
    for i, src in enumerate(sources):
        src = parse_source(src) if isinstance(src, str) else src
        files = src.files or list_token_files(src.prefix, extension)
        available = sum(size // bytes_per_token for _, size in files)
        rng = random.Random(f"{seed}:{i}:{src.prefix}")
        chosen: List[Tuple[str, int]] = []
        if src.repeat is not None:
            whole, part = int(src.repeat), src.repeat - int(src.repeat)
            for _ in range(whole):
                chosen += sorted(files)
            if part > 0:
                chosen += select_files(files, available * part, bytes_per_token, rng)
        else:
            target = src.tokens if src.tokens is not None else available * (src.fraction if src.fraction is not None else 1.0)
            if target > available:
                raise ValueError(f"source {src.prefix} holds {human_count(available)} tokens, {human_count(target)} were asked for; "
                                 "use repeat to take it more than once")
            chosen = sorted(files) if target >= available else select_files(files, target, bytes_per_token, rng)
        paths += [p for p, _ in chosen]
        rows.append({"source": src.name or src.prefix, "files": len(chosen), "tokens": sum(s // bytes_per_token for _, s in chosen),
                     "available": available})
    total = sum(int(r["tokens"]) for r in rows) or 1
    for r in rows:
        r["share"] = int(r["tokens"]) / total
    return paths, rows


def examine(paths: Sequence[str], *, bytes_per_token: int = 4, depth: int = 1, threads: int = 16) -> List[Dict[str, object]]:
    """Tokens per source of an existing path list; a source is a path's parent folder, ``depth`` levels up."""
    with ThreadPoolExecutor(max_workers=threads) as pool:
        sizes = list(pool.map(file_size, paths))
    groups: Dict[str, List[int]] = {}
    for path, size in zip(paths, sizes):
        key = str(path).rstrip("/")
        for _ in range(depth):
            key = key.rsplit("/", 1)[0]
        groups.setdefault(key, []).append(size // bytes_per_token)
    total = sum(sum(v) for v in groups.values()) or 1
    return [{"source": k, "files": len(v), "tokens": sum(v), "share": sum(v) / total} for k, v in sorted(groups.items())]


def human_count(n: float) -> str:
    """``1234567`` -> ``1.23M``."""
    for limit, suffix in ((1e12, "T"), (1e9, "B"), (1e6, "M"), (1e3, "K")):
        if abs(n) >= limit:
            return f"{n / limit:.2f}{suffix}"
    return f"{n:.0f}"
