#!/usr/bin/env python
"""Split gzip-compressed line files (JSON lines) into smaller gzip files, by lines or by uncompressed size.

    scripts/split_gz.py --input_dir IN --output_dir OUT [--input_ext .gz] [--output_ext .gz] [--size_limit BYTES] [--lines N]
    scripts/split_gz.py IN.json.gz OUT_PREFIX [--lines 100000] [--size_limit BYTES]

Directory form (the options of the reference's ``scripts/split_gz.py``): every ``*INPUT_EXT`` file of ``IN`` becomes
``OUT/<name>_0000OUTPUT_EXT``, ``…_0001…``; files are processed in parallel by worker threads (zlib releases the interpreter lock).
A part is closed before the line that would take it past ``--size_limit`` bytes of text (default 4 GiB) or ``--lines`` lines.
"""
import argparse
import gzip
import os
import sys
from concurrent.futures import ThreadPoolExecutor
from typing import List, Optional

FOUR_GIB = 4 * 1024 * 1024 * 1024


def split_file(source: str, output_base: str, output_ext: str = ".gz", size_limit: int = FOUR_GIB, lines: Optional[int] = None) -> List[str]:
    """Write ``source`` as ``<output_base>_0000<ext>``, ``_0001`` … and return the paths."""
    written: List[str] = []
    out = None
    size = count = 0
    with gzip.open(source, "rt") as f:
        for line in f:
            full = out is not None and (size + len(line) > size_limit or (lines is not None and count >= lines))
            if out is None or full:
                if out is not None:
                    out.close()
                written.append(f"{output_base}_{len(written):04d}{output_ext}")
                out = gzip.open(written[-1], "wt")
                size = count = 0
            out.write(line)
            size += len(line)
            count += 1
    if out is not None:
        out.close()
    return written


def _job(args) -> List[str]:
    return split_file(*args)


def split_directory(input_dir: str, output_dir: str, input_ext: str = ".gz", output_ext: str = ".gz", size_limit: int = FOUR_GIB,
                    lines: Optional[int] = None, workers: Optional[int] = None) -> List[str]:
    os.makedirs(output_dir, exist_ok=True)
    jobs = []
    for name in sorted(os.listdir(input_dir)):
        path = os.path.join(input_dir, name)
        if name.endswith(input_ext) and os.path.isfile(path):
            jobs.append((path, os.path.join(output_dir, name[: -len(input_ext)] if input_ext else name), output_ext, size_limit, lines))
    if len(jobs) <= 1 or workers == 1:
        parts = [_job(j) for j in jobs]
    else:
        with ThreadPoolExecutor(max_workers=workers) as pool:
            parts = list(pool.map(_job, jobs))
    return [p for group in parts for p in group]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("input", nargs="?", help="one input file (single-file form)")
    ap.add_argument("prefix", nargs="?", help="output prefix (single-file form)")
    ap.add_argument("--input_dir", default=None)
    ap.add_argument("--output_dir", default=None)
    ap.add_argument("--input_ext", default=".gz")
    ap.add_argument("--output_ext", default=".gz")
    ap.add_argument("--size_limit", type=int, default=FOUR_GIB, help="bytes of text per part")
    ap.add_argument("--lines", type=int, default=None, help="lines per part")
    ap.add_argument("--workers", type=int, default=None)
    a = ap.parse_args(argv)
    if a.input_dir is not None:
        if a.output_dir is None:
            ap.error("--output_dir is required with --input_dir")
        written = split_directory(a.input_dir, a.output_dir, a.input_ext, a.output_ext, a.size_limit, a.lines, a.workers)
    elif a.input and a.prefix:
        written = split_file(a.input, a.prefix, ".json.gz", a.size_limit, a.lines if a.lines is not None else 100_000)
    else:
        ap.error("give --input_dir/--output_dir, or an input file and an output prefix")
    print(f"{len(written)} parts")
    return len(written)


if __name__ == "__main__":
    sys.exit(0 if main() >= 0 else 1)
