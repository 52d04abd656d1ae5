#!/usr/bin/env python
"""Split a gzip'd JSON-lines file into parts of at most N lines each: ``split_gz.py IN.json.gz OUT_PREFIX --lines 100000``
(reference: ``scripts/split_gz.py``)."""
import argparse
import gzip

if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("input")
    ap.add_argument("prefix")
    ap.add_argument("--lines", type=int, default=100_000)
    a = ap.parse_args()
    part, count, out = 0, 0, None
    with gzip.open(a.input, "rt") as f:
        for line in f:
            if out is None or count >= a.lines:
                if out is not None:
                    out.close()
                out = gzip.open(f"{a.prefix}.{part:04d}.json.gz", "wt")
                part, count = part + 1, 0
            out.write(line)
            count += 1
    if out is not None:
        out.close()
    print(f"{part} parts")
