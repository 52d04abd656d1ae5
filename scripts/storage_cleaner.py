#!/usr/bin/env python
"""Housekeeping for run folders on any storage backend the framework can address (local paths, ``s3://``, ``r2://``,
``weka://``, ``gs://``):

* ``clean``    delete runs that never produced a checkpoint (or whose newest checkpoint is older than a step bound);
* ``unshard``  convert the sharded checkpoints of a run into unsharded ones next to them;
* ``move``     copy a run (or a single checkpoint) to another location, optionally keeping only the latest K checkpoints.

The reference's ``scripts/storage_cleaner.py`` implements its own storage adapters; here the operations are expressed on
the framework's :class:`olmo_b200.util.StorageBackend` interface (``list_files`` / ``file_size`` / ``get_bytes_range`` /
``upload`` / ``delete``), so a new backend registered there is automatically supported.

    python scripts/storage_cleaner.py clean  RUNS_ROOT [--max-step-without-checkpoint 0] [--dry-run]
    python scripts/storage_cleaner.py unshard RUN_DIR [--latest-only] [--safe-tensors]
    python scripts/storage_cleaner.py move   SRC DST [--keep-latest K] [--dry-run]
"""
from __future__ import annotations

import argparse
import logging
import re
import shutil
import sys
import tempfile
from pathlib import Path
from typing import List, Optional, Tuple

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from olmo_b200.util import delete_file, file_size, get_bytes_range, is_url, list_files, upload  # noqa: E402

log = logging.getLogger("storage_cleaner")
_STEP = re.compile(r"^step(\d+)(-unsharded)?$")


def list_dir(location: str) -> List[str]:
    """Immediate children (names only) of a local folder or a remote prefix."""
    if not is_url(location):
        p = Path(location)
        return sorted(c.name for c in p.iterdir()) if p.is_dir() else []
    names = set()
    prefix = location.rstrip("/") + "/"
    for key in list_files(prefix):
        rest = key[len(prefix) :] if key.startswith(prefix) else key
        if rest:
            names.add(rest.split("/", 1)[0])
    return sorted(names)


def checkpoints_of(run: str) -> List[Tuple[int, bool, str]]:
    out = []
    for name in list_dir(run):
        m = _STEP.match(name)
        if m:
            out.append((int(m.group(1)), m.group(2) is not None, f"{run.rstrip('/')}/{name}"))
    return sorted(out)


def delete_tree(location: str, dry_run: bool) -> None:
    log.info("%sdelete %s", "[dry run] " if dry_run else "", location)
    if dry_run:
        return
    if not is_url(location):
        shutil.rmtree(location, ignore_errors=True)
    else:
        for key in list_files(location.rstrip("/") + "/"):
            delete_file(key)


def copy_tree(src: str, dst: str, dry_run: bool) -> int:
    """Copy every file below ``src`` to the same relative place below ``dst``; returns the number of files."""
    files: List[Tuple[str, str]] = []
    if not is_url(src):
        base = Path(src)
        files = [(str(p), p.relative_to(base).as_posix()) for p in sorted(base.rglob("*")) if p.is_file()]
    else:
        prefix = src.rstrip("/") + "/"
        files = [(k, k[len(prefix) :]) for k in list_files(prefix)]
    for full, rel in files:
        target = f"{dst.rstrip('/')}/{rel}"
        log.info("%scopy %s -> %s", "[dry run] " if dry_run else "", full, target)
        if dry_run:
            continue
        if is_url(full):
            with tempfile.NamedTemporaryFile(delete=False) as tmp:
                size, chunk = file_size(full), 64 << 20
                for off in range(0, size, chunk):
                    tmp.write(get_bytes_range(full, off, min(chunk, size - off)))
            local = Path(tmp.name)
        else:
            local = Path(full)
        if is_url(target):
            upload(local, target, save_overwrite=True)
        else:
            Path(target).parent.mkdir(parents=True, exist_ok=True)
            shutil.copyfile(local, target)
        if is_url(full):
            local.unlink(missing_ok=True)
    return len(files)


def clean(root: str, max_step: int, dry_run: bool) -> List[str]:
    removed = []
    for name in list_dir(root):
        run = f"{root.rstrip('/')}/{name}"
        if "config.yaml" not in list_dir(run) and not checkpoints_of(run):
            continue  # not a run folder
        ckpts = checkpoints_of(run)
        newest = ckpts[-1][0] if ckpts else -1
        if newest <= max_step:
            delete_tree(run, dry_run)
            removed.append(run)
    return removed


def unshard_run(run: str, latest_only: bool, safe_tensors: bool) -> List[str]:
    from unshard import main as unshard
    from olmo_b200.config import TrainConfig

    if is_url(run):
        raise SystemExit("unshard works on local folders: `move` the run to local storage first")
    done = []
    ckpts = [(s, path) for s, unsharded, path in checkpoints_of(run) if not unsharded]
    have = {s for s, unsharded, _ in checkpoints_of(run) if unsharded}
    if latest_only:
        ckpts = ckpts[-1:]
    for step, path in ckpts:
        if step in have:
            continue
        cfg = TrainConfig.load(Path(path) / "config.yaml", validate_paths=False)
        out = f"{run.rstrip('/')}/step{step}-unsharded"
        unshard(path, out, sharded_checkpoint_type=cfg.sharded_checkpointer, safe_tensors=safe_tensors)
        done.append(out)
    return done


def move(src: str, dst: str, keep_latest: Optional[int], dry_run: bool) -> int:
    ckpts = checkpoints_of(src)
    if not ckpts or keep_latest is None:
        return copy_tree(src, dst, dry_run)
    steps = sorted({s for s, _, _ in ckpts})[-keep_latest:]
    n = 0
    for name in list_dir(src):
        m = _STEP.match(name)
        if m and int(m.group(1)) not in steps:
            continue
        child = f"{src.rstrip('/')}/{name}"
        if not is_url(child) and Path(child).is_file():
            if not dry_run:
                Path(dst).mkdir(parents=True, exist_ok=True) if not is_url(dst) else None
                (shutil.copyfile(child, f"{dst.rstrip('/')}/{name}") if not is_url(dst) else upload(Path(child), f"{dst.rstrip('/')}/{name}", save_overwrite=True))
            n += 1
        else:
            n += copy_tree(child, f"{dst.rstrip('/')}/{name}", dry_run)
    return n


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("clean")
    p.add_argument("root")
    p.add_argument("--max-step-without-checkpoint", type=int, default=0, help="runs whose newest checkpoint step is <= this are deleted")
    p.add_argument("--dry-run", action="store_true")
    p = sub.add_parser("unshard")
    p.add_argument("run")
    p.add_argument("--latest-only", action="store_true")
    p.add_argument("--safe-tensors", action="store_true")
    p = sub.add_parser("move")
    p.add_argument("src")
    p.add_argument("dst")
    p.add_argument("--keep-latest", type=int, default=None)
    p.add_argument("--dry-run", action="store_true")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    if args.cmd == "clean":
        return len(clean(args.root, args.max_step_without_checkpoint, args.dry_run))
    if args.cmd == "unshard":
        return len(unshard_run(args.run, args.latest_only, args.safe_tensors))
    return move(args.src, args.dst, args.keep_latest, args.dry_run)


if __name__ == "__main__":
    main()
