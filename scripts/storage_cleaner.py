#!/usr/bin/env python
"""Housekeeping for run folders on any storage backend the framework can address (local paths, ``s3://``, ``r2://``,
``weka://``, ``gs://``):

* ``clean``    delete runs that never produced a checkpoint (or whose newest checkpoint is older than a step bound);
* ``unshard``  convert the sharded checkpoints of a run into unsharded ones next to them;
* ``move``     copy a run (or a single checkpoint) to another location, optionally keeping only the latest K checkpoints.

The reference's ``scripts/storage_cleaner.py`` implements its own storage adapters; here the operations are expressed on
the framework's :class:`olmo_b200.util.StorageBackend` interface (``list_files`` / ``file_size`` / ``get_bytes_range`` /
``upload`` / ``delete``), so a new backend registered there is automatically supported.

A run may also be an archive file (``.tar``, ``.tar.gz``, ``.tgz``, ``.zip``) of a run folder: ``clean`` inspects and deletes
archives (up to ``--max-archive-size``), ``unshard`` and ``move --store-unarchived`` unpack them into ``--temp-dir`` first.

    python scripts/storage_cleaner.py clean  RUNS_ROOT [--max-step-without-checkpoint 0] [--ignore-non-runs | --skip-run-verification]
                                             [--max-archive-size BYTES] [--dry-run]
    python scripts/storage_cleaner.py unshard RUN [DEST_DIR] [--latest-only] [--checkpoint-num N] [--delete-sharded] [--safe-tensors]
    python scripts/storage_cleaner.py move   SRC DST [--keep-latest K] [--entry NAME] [--keep-src] [--store-unarchived]
                                             [--append-wandb-path] [--dry-run]
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


_ARCHIVE_SUFFIXES = (".tar", ".tar.gz", ".tgz", ".zip")


def is_archive(location: str) -> bool:
    return location.lower().endswith(_ARCHIVE_SUFFIXES)


def fetch_local(location: str, temp_dir: Optional[str]) -> Path:
    """A local copy of one remote file (the file itself when it is local already)."""
    if not is_url(location):
        return Path(location)
    target = Path(tempfile.mkdtemp(dir=temp_dir)) / location.rstrip("/").rsplit("/", 1)[-1]
    size, chunk = file_size(location), 64 << 20
    with open(target, "wb") as f:
        for off in range(0, size, chunk):
            f.write(get_bytes_range(location, off, min(chunk, size - off)))
    return target


def unpack_archive(location: str, temp_dir: Optional[str]) -> str:
    """Unpack an archived run into a temporary folder and return the run folder inside it (archives hold either the run's
    files directly or one top-level folder)."""
    local = fetch_local(location, temp_dir)
    out = Path(tempfile.mkdtemp(dir=temp_dir))
    if str(local).lower().endswith(".zip"):
        shutil.unpack_archive(str(local), str(out))
    else:
        shutil.unpack_archive(str(local), str(out), filter="data")  # no absolute paths, links out of the tree or device files
    children = [c for c in out.iterdir()]
    return str(children[0]) if len(children) == 1 and children[0].is_dir() else str(out)


def archive_entries(location: str, temp_dir: Optional[str]) -> List[str]:
    """Top-level names inside an archived run, without unpacking it."""
    import tarfile
    import zipfile

    local = fetch_local(location, temp_dir)
    if str(local).lower().endswith(".zip"):
        with zipfile.ZipFile(local) as z:
            names = z.namelist()
    else:
        with tarfile.open(local) as t:
            names = t.getnames()
    parts = [n.strip("/").split("/") for n in names if n.strip("/")]
    tops = {p[0] for p in parts}
    if len(tops) == 1 and any(len(p) > 1 for p in parts):  # one wrapping folder: look inside it
        return sorted({p[1] for p in parts if len(p) > 1})
    return sorted(tops)


def looks_like_run(entries: List[str]) -> bool:
    """A run folder holds its config, checkpoints, or the trainer's side products."""
    return "config.yaml" in entries or any(_STEP.match(e) for e in entries) or any(e in ("wandb", "train_data", "data-indices") for e in entries)


def clean(root: str, max_step: int, dry_run: bool, ignore_non_runs: bool = True, skip_run_verification: bool = False,
          max_archive_size: Optional[int] = None, temp_dir: Optional[str] = None) -> List[str]:
    """Delete the runs below ``root`` whose newest checkpoint step is at most ``max_step`` (runs that never got anywhere).
    Entries that do not look like runs are skipped (``ignore_non_runs``), refused with an error, or — with
    ``skip_run_verification`` — treated as runs."""
    removed = []
    for name in list_dir(root):
        run = f"{root.rstrip('/')}/{name}"
        if is_archive(run):
            if max_archive_size is not None and file_size(run) > max_archive_size:
                log.info("skip %s: archive larger than %d bytes", run, max_archive_size)
                continue
            entries = archive_entries(run, temp_dir)
        else:
            entries = list_dir(run)
        if not skip_run_verification and not looks_like_run(entries):
            if ignore_non_runs:
                continue
            raise SystemExit(f"{run} does not look like a run (no config.yaml, checkpoints, wandb or train_data); "
                             "pass --ignore-non-runs to skip such entries or --skip-run-verification to delete them anyway")
        steps = [int(m.group(1)) for m in (_STEP.match(e) for e in entries) if m]
        newest = max(steps) if steps else -1
        if newest <= max_step:
            if is_archive(run):
                log.info("%sdelete %s", "[dry run] " if dry_run else "", run)
                if not dry_run:
                    delete_file(run) if is_url(run) else Path(run).unlink()
            else:
                delete_tree(run, dry_run)
            removed.append(run)
    return removed


def unshard_run(run: str, latest_only: bool, safe_tensors: bool, dest: Optional[str] = None, checkpoint_num: Optional[int] = None,
                delete_sharded: bool = False, temp_dir: Optional[str] = None) -> List[str]:
    """Unshard the sharded checkpoints of a run (a folder, an archive, or a remote prefix, which is copied to ``temp_dir``
    first).  Results go next to the sharded ones, or into ``dest`` (only the unsharded checkpoints are stored there)."""
    from unshard import main as unshard
    from olmo_b200.config import TrainConfig

    if is_archive(run):
        run = unpack_archive(run, temp_dir)
        if dest is None:
            raise SystemExit("unsharding an archived run needs a destination folder for the results")
    elif is_url(run):
        local = tempfile.mkdtemp(dir=temp_dir)
        copy_tree(run, local, dry_run=False)
        if dest is None:
            dest = run  # results are uploaded back next to the sharded checkpoints
        run = local
    done = []
    ckpts = [(s, path) for s, unsharded, path in checkpoints_of(run) if not unsharded]
    have = {s for s, unsharded, _ in checkpoints_of(run) if unsharded}
    if checkpoint_num is not None:
        ckpts = [c for c in ckpts if c[0] == checkpoint_num]
        if not ckpts:
            raise SystemExit(f"the run has no sharded checkpoint for step {checkpoint_num}")
    if latest_only:
        ckpts = ckpts[-1:]
    for step, path in ckpts:
        if step in have and dest is None:
            continue
        cfg = TrainConfig.load(Path(path) / "config.yaml", validate_paths=False)
        name = f"step{step}-unsharded"
        local_out = f"{run.rstrip('/')}/{name}" if dest is None or is_url(dest) else f"{dest.rstrip('/')}/{name}"
        unshard(path, local_out, sharded_checkpoint_type=cfg.sharded_checkpointer, safe_tensors=safe_tensors)
        if dest is not None and is_url(dest):
            copy_tree(local_out, f"{dest.rstrip('/')}/{name}", dry_run=False)
        done.append(local_out if dest is None or not is_url(dest) else f"{dest.rstrip('/')}/{name}")
        if delete_sharded:
            delete_tree(path, dry_run=False)
    return done


def wandb_path_of(run: str) -> Optional[str]:
    """``entity/project/group/name`` style path of the run's W&B record, read from its saved config (``wandb`` section)."""
    import yaml

    cfg_file = Path(run) / "config.yaml"
    if is_url(run) or not cfg_file.is_file():
        return None
    wandb = (yaml.safe_load(cfg_file.read_text()) or {}).get("wandb") or {}
    parts = [wandb.get(k) for k in ("entity", "project", "group", "name")]
    parts = [str(x) for x in parts if x]
    return "/".join(parts) if parts else None


def move(src: str, dst: str, keep_latest: Optional[int], dry_run: bool, keep_src: bool = True, entry: Optional[str] = None,
         store_unarchived: bool = False, append_wandb_path: bool = False, temp_dir: Optional[str] = None) -> int:
    """Copy a run (or one ``entry`` of it, e.g. ``step0-unsharded``) to ``dst``; with ``keep_src=False`` the source is
    removed afterwards (a true move).  Archives are moved as files unless ``store_unarchived``."""
    archived = is_archive(src)
    if archived and (store_unarchived or entry is not None or append_wandb_path):
        work = unpack_archive(src, temp_dir)
    else:
        work = src
    if append_wandb_path:
        extra = wandb_path_of(work)
        if extra is None:
            raise SystemExit("--append-wandb-path needs a local run (or archive) whose config.yaml has a wandb section")
        dst = f"{dst.rstrip('/')}/{extra}"
    if archived and work == src:  # the archive file itself
        name = src.rstrip("/").rsplit("/", 1)[-1]
        log.info("%scopy %s -> %s/%s", "[dry run] " if dry_run else "", src, dst, name)
        if not dry_run:
            local = fetch_local(src, temp_dir)
            if is_url(dst):
                upload(local, f"{dst.rstrip('/')}/{name}", save_overwrite=True)
            else:
                Path(dst).mkdir(parents=True, exist_ok=True)
                shutil.copyfile(local, f"{dst.rstrip('/')}/{name}")
        n = 1
    elif entry is not None:
        child = f"{work.rstrip('/')}/{entry}"
        if not is_url(child) and Path(child).is_file():
            if not dry_run:
                if is_url(dst):
                    upload(Path(child), f"{dst.rstrip('/')}/{entry}", save_overwrite=True)
                else:
                    Path(dst).mkdir(parents=True, exist_ok=True)
                    shutil.copyfile(child, f"{dst.rstrip('/')}/{entry}")
            n = 1
        else:
            n = copy_tree(child, f"{dst.rstrip('/')}/{entry}", dry_run)
            if n == 0:
                raise SystemExit(f"{src} has no entry named {entry}")
    else:
        n = _copy_run(work, dst, keep_latest, dry_run)
    if not keep_src and not dry_run:
        if archived:
            delete_file(src) if is_url(src) else Path(src).unlink()
        else:
            delete_tree(src if entry is None else f"{src.rstrip('/')}/{entry}", dry_run=False)
    return n


def _copy_run(src: str, dst: str, keep_latest: Optional[int], dry_run: bool) -> int:
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
    ap.add_argument("--temp-dir", default=None, help="local folder for temporary copies and unpacked archives")
    p = sub.add_parser("clean", help="delete runs that never produced a useful checkpoint")
    p.add_argument("root", help="folder (or remote prefix) whose children are run folders or run archives")
    p.add_argument("--max-step-without-checkpoint", type=int, default=0, help="runs whose newest checkpoint step is <= this are deleted")
    g = p.add_mutually_exclusive_group()
    g.add_argument("--ignore-non-runs", action="store_true", default=True, help="skip entries that do not look like runs (default)")
    g.add_argument("--fail-on-non-runs", dest="ignore_non_runs", action="store_false", help="stop at the first entry that does not look like a run")
    g.add_argument("--skip-run-verification", "--bypass_run_verification", dest="skip_run_verification", action="store_true",
                   help="(unsafe) treat every entry as a run")
    p.add_argument("--max-archive-size", type=int, default=None, help="archives larger than this many bytes are left alone")
    p.add_argument("--dry-run", action="store_true")
    p = sub.add_parser("unshard", help="unshard the checkpoints of a run")
    p.add_argument("run", help="run folder, run archive or remote prefix")
    p.add_argument("dest", nargs="?", default=None, help="where the unsharded checkpoints go (default: next to the sharded ones)")
    p.add_argument("--latest-only", "--latest_checkpoint_only", dest="latest_only", action="store_true", help="only the newest sharded checkpoint")
    p.add_argument("--checkpoint-num", type=int, default=None, help="only the checkpoint of this step")
    p.add_argument("--delete-sharded", action="store_true", help="remove a sharded checkpoint once it has been unsharded")
    p.add_argument("--safe-tensors", action="store_true")
    p = sub.add_parser("move", help="copy or move a run")
    p.add_argument("src")
    p.add_argument("dst")
    p.add_argument("--keep-latest", type=int, default=None, help="only the newest K checkpoints (and all non-checkpoint files)")
    p.add_argument("--entry", default=None, help="only this folder or file of the run, e.g. step0-unsharded")
    p.add_argument("--keep-src", action="store_true", default=True, help="leave the source in place (default)")
    p.add_argument("--remove-src", dest="keep_src", action="store_false", help="delete the source after the copy")
    p.add_argument("--store-unarchived", "--unarchive", dest="store_unarchived", action="store_true",
                   help="an archived run is stored unpacked at the destination")
    p.add_argument("--append-wandb-path", action="store_true", help="append entity/project/group/name from the run's config to DST")
    p.add_argument("--dry-run", action="store_true")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    if args.cmd == "clean":
        return len(clean(args.root, args.max_step_without_checkpoint, args.dry_run, ignore_non_runs=args.ignore_non_runs,
                         skip_run_verification=args.skip_run_verification, max_archive_size=args.max_archive_size, temp_dir=args.temp_dir))
    if args.cmd == "unshard":
        return len(unshard_run(args.run, args.latest_only, args.safe_tensors, dest=args.dest, checkpoint_num=args.checkpoint_num,
                               delete_sharded=args.delete_sharded, temp_dir=args.temp_dir))
    return move(args.src, args.dst, args.keep_latest, args.dry_run, keep_src=args.keep_src, entry=args.entry,
                store_unarchived=args.store_unarchived, append_wandb_path=args.append_wandb_path, temp_dir=args.temp_dir)


if __name__ == "__main__":
    main()
