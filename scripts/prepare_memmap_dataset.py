#!/usr/bin/env python
"""Tokenise ``{"text": ...}`` JSON-lines documents (plain or gzip) into flat ``.npy`` token files that
:class:`olmo_b200.data.MemMapDataset` reads: every document is followed by the EOS id; a new output file starts whenever
``--max-tokens`` would be exceeded (reference: ``scripts/prepare_memmap_dataset.py``, which upstream marks as deprecated
in favour of the Dolma toolkit's tokeniser — the file format is the same).

    python scripts/prepare_memmap_dataset.py SRC [SRC ...] -o OUT_DIR --tokenizer tok.json [--dtype uint16] [--workers 8] [--validate]
"""
from __future__ import annotations

import argparse
import concurrent.futures
import gzip
import json
import logging
import os
import random
import sys
from pathlib import Path
from typing import Iterator, List, Optional, Sequence, Tuple

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np

log = logging.getLogger("prepare_memmap_dataset")


_DOC_SUFFIXES = ("gz", "json", "jsonl")

#: where remote sources are copied before they are read (``--cache-dir``; a temporary folder when unset)
_CACHE_DIR: Optional[str] = None


def list_sources(prefixes: Sequence[str]) -> List[str]:
    """Document files below local folders or remote prefixes (any storage scheme the framework knows)."""
    from olmo_b200.util import is_url, list_files

    out: List[str] = []
    for prefix in prefixes:
        if is_url(prefix):
            found = [u for u in list_files(prefix) if u.rsplit(".", 1)[-1] in _DOC_SUFFIXES]
            if not found:
                found = [prefix]  # a single remote file
            out.extend(found)
            continue
        p = Path(prefix)
        if p.is_dir():
            out.extend(sorted(str(q) for q in p.rglob("*") if q.is_file() and q.name.split(".")[-1] in _DOC_SUFFIXES))
        elif p.is_file():
            out.append(str(p))
        else:
            raise FileNotFoundError(prefix)
    return out


def local_copy(source: str) -> Path:
    """The file itself when it is local; otherwise a copy in the cache folder (kept, so a rerun does not fetch it again)."""
    from olmo_b200.util import file_size, get_bytes_range, is_url

    if not is_url(source):
        return Path(source)
    import hashlib
    import tempfile

    root = Path(_CACHE_DIR or tempfile.gettempdir()) / "prepare_memmap_cache"
    root.mkdir(parents=True, exist_ok=True)
    target = root / (hashlib.sha256(source.encode()).hexdigest()[:16] + "-" + source.rstrip("/").rsplit("/", 1)[-1])
    size = file_size(source)
    if not target.is_file() or target.stat().st_size != size:
        tmp = target.with_suffix(target.suffix + f".part{os.getpid()}")
        with open(tmp, "wb") as f:
            for off in range(0, size, 64 << 20):
                f.write(get_bytes_range(source, off, min(64 << 20, size - off)))
        os.replace(tmp, target)
    return target


def read_documents(path) -> Iterator[str]:
    path = local_copy(str(path))
    opener = gzip.open if path.suffix == ".gz" else open
    with opener(path, "rt", encoding="utf-8") as f:
        for line in f:
            line = line.strip()
            if line:
                yield json.loads(line)["text"]


def load_tokenizer(identifier: str, eos_token_id=None):
    from olmo_b200.tokenizer import Tokenizer

    kwargs = {} if eos_token_id is None else {"eos_token_id": eos_token_id}
    if Path(identifier).is_file():
        return Tokenizer.from_file(identifier, **kwargs)
    return Tokenizer.from_pretrained(identifier, **kwargs)


class MemmapWriter:
    """Append-only token file; the array is created at ``max_tokens`` and trimmed on close."""

    def __init__(self, path: Path, dtype: np.dtype, max_tokens: int):
        self.path, self.dtype, self.max_tokens = path, dtype, max_tokens
        path.parent.mkdir(parents=True, exist_ok=True)
        self.array = np.memmap(path, mode="w+", dtype=dtype, shape=(max_tokens,))
        self.used = 0

    def fits(self, n: int) -> bool:
        return self.used + n <= self.max_tokens

    def write(self, ids: Sequence[int]) -> None:
        self.array[self.used : self.used + len(ids)] = ids
        self.used += len(ids)

    def close(self) -> int:
        self.array.flush()
        del self.array
        with open(self.path, "r+b") as f:
            f.truncate(self.used * self.dtype.itemsize)
        return self.used


def fill(job: Tuple[List[str], str, str, str, int, float, int, int, object, Optional[str]]) -> int:
    global _CACHE_DIR
    sources, out_stem, tokenizer_id, dtype_str, max_tokens, sample_rate, seed, repeat, eos, _CACHE_DIR = job
    tok = load_tokenizer(tokenizer_id, eos)
    dtype = np.dtype(dtype_str)
    limit = np.iinfo(dtype).max
    rng = random.Random(seed)
    part, total = 0, 0
    writer = MemmapWriter(Path(f"{out_stem}_{part:05d}.npy"), dtype, max_tokens)
    for src in sources:
        for text in read_documents(src):
            if sample_rate < 1.0 and rng.random() > sample_rate:
                continue
            ids = tok.encode(text, add_special_tokens=True)
            if ids and max(ids) > limit:
                raise ValueError(f"token id {max(ids)} does not fit {dtype_str}")
            for _ in range(repeat):
                if len(ids) > max_tokens:
                    raise ValueError("a single document is longer than --max-tokens")
                if not writer.fits(len(ids)):
                    total += writer.close()
                    part += 1
                    writer = MemmapWriter(Path(f"{out_stem}_{part:05d}.npy"), dtype, max_tokens)
                writer.write(ids)
    total += writer.close()
    return total


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("src", nargs="+")
    ap.add_argument("-o", "--output", required=True)
    ap.add_argument("--tokenizer", "--tokenizer-id", dest="tokenizer", required=True, help="tokenizer.json path or HF Hub name")
    ap.add_argument("--eos-token-id", type=int, default=None)
    ap.add_argument("--dtype", default="uint16", choices=["uint8", "uint16", "uint32", "uint64"])
    ap.add_argument("--max-tokens", type=int, default=512 * 1024 * 1024)
    ap.add_argument("--sample-rate", type=float, default=1.0)
    ap.add_argument("--random-seed", type=int, default=3920)
    ap.add_argument("--repeat-sequence", type=int, default=1)
    ap.add_argument("--paths-per-worker", type=int, default=1)
    ap.add_argument("--workers", "--max-workers", dest="workers", type=int, default=1)
    ap.add_argument("--validate", action="store_true")
    ap.add_argument("--ack-deprecated", action="store_true", help="accepted for command-line compatibility")
    ap.add_argument("--cache-dir", default=None, help="where remote source files are copied before they are read (kept for reruns)")
    ap.add_argument("--safe-mode", action="store_true", help="accepted for compatibility: remote files are always copied before they are read")
    args = ap.parse_args(argv)
    global _CACHE_DIR
    _CACHE_DIR = args.cache_dir
    logging.basicConfig(level=logging.INFO)

    sources = list_sources(args.src)
    random.Random(args.random_seed).shuffle(sources)
    groups = [sources[i : i + args.paths_per_worker] for i in range(0, len(sources), args.paths_per_worker)]
    out = Path(args.output)
    jobs = [
        ([str(s) for s in group], str(out / f"part-{i:03d}"), args.tokenizer, args.dtype, args.max_tokens, args.sample_rate,
         args.random_seed + i, args.repeat_sequence, args.eos_token_id, args.cache_dir)
        for i, group in enumerate(groups)
    ]
    if args.workers <= 1 or len(jobs) == 1:
        total = sum(fill(j) for j in jobs)
    else:
        with concurrent.futures.ProcessPoolExecutor(max_workers=min(args.workers, len(jobs))) as pool:
            total = sum(pool.map(fill, jobs))
    log.info("wrote %s tokens under %s", f"{total:,}", out)

    if args.validate:
        tok = load_tokenizer(args.tokenizer, args.eos_token_id)
        want_tokens = want_docs = 0
        for src in sources:
            for text in read_documents(src):
                want_docs += 1
                want_tokens += len(tok.encode(text, add_special_tokens=True))
        for f in sorted(out.rglob("*.npy")):
            arr = np.memmap(f, mode="r", dtype=np.dtype(args.dtype))
            want_tokens -= len(arr) // args.repeat_sequence if args.repeat_sequence > 1 else len(arr)
            want_docs -= int((arr == tok.eos_token_id).sum()) // args.repeat_sequence if args.repeat_sequence > 1 else int((arr == tok.eos_token_id).sum())
            assert (arr < tok.vocab_size).all(), f"invalid token id in {f}"
        if args.sample_rate >= 1.0:
            assert want_tokens == 0, f"token count mismatch: {want_tokens}"
            assert want_docs == 0, f"document count mismatch: {want_docs}"
        log.info("validation passed")
    return total


if __name__ == "__main__":
    main()
