#!/usr/bin/env python
"""Remote sharded checkpoint -> local copy -> unsharded -> HuggingFace directory -> upload.  Works with every storage scheme
the framework addresses (s3, r2, weka, gs, local), through its own storage layer instead of the ``aws`` command line.

    python scripts/s3_unshard_to_hf.py --sharded_bucket s3://bucket/run/step1000 --hf_bucket s3://bucket/run/step1000-hf \\
        [--unsharded_bucket s3://bucket/run/step1000-unsharded] [--checkpoint_style transformers|hf_olmo] [--local_dir /scratch]
        [--already_downloaded] [--already_unsharded] [--model_only] [--type torch_legacy] [--cleanup_local_dir] [--quiet]

The option names are those of the reference's ``scripts/s3_unshard_to_hf.py:28-76`` (``--sharded-url``, ``--unsharded-url``,
``--hf-url``, ``--layout``, ``--tmp-dir`` are accepted as other spellings).  Inside ``--local_dir`` the three stages live in
``sharded/``, ``unsharded/`` and ``hf/``, so a run that was interrupted can continue with ``--already_downloaded`` or
``--already_unsharded``.
"""
import argparse
import logging
import shutil
import sys
import tempfile
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
sys.path.insert(0, str(Path(__file__).resolve().parent))

log = logging.getLogger("s3_unshard_to_hf")


def make_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--sharded_bucket", "--sharded-url", dest="sharded", default=None, help="where the sharded checkpoint is")
    ap.add_argument("--unsharded_bucket", "--unsharded-url", dest="unsharded", default=None, help="also keep the unsharded checkpoint here")
    ap.add_argument("--hf_bucket", "--hf-url", dest="hf", default=None, help="where the converted checkpoint goes")
    ap.add_argument("--already_downloaded", action="store_true", help="the sharded checkpoint is in LOCAL_DIR/sharded already")
    ap.add_argument("--already_unsharded", action="store_true", help="LOCAL_DIR/unsharded (or --unsharded_bucket) holds the unsharded checkpoint: only convert")
    ap.add_argument("--local_dir", "--tmp-dir", dest="local_dir", default=None, help="working folder (default: a temporary one)")
    ap.add_argument("--cleanup_local_dir", action="store_true", help="remove the working folder after a successful run")
    ap.add_argument("--checkpoint_style", "--layout", dest="style", choices=["hf_olmo", "transformers"], default="hf_olmo")
    ap.add_argument("--hf_olmo", action="store_true", help="same as --checkpoint_style hf_olmo")
    ap.add_argument("--quiet", action="store_true", help="log warnings only")
    ap.add_argument("--type", default=None, help="sharded layout to expect (checked against what is found; see scripts/unshard.py)")
    ap.add_argument("--model_only", action="store_true", help="unshard the weights only")
    ap.add_argument("--tokenizer", default=None, help="tokenizer.json to ship instead of the configured one")
    return ap


def main(argv=None) -> str:
    args = make_parser().parse_args(argv)
    logging.basicConfig(level=logging.WARNING if args.quiet else logging.INFO, format="%(message)s")
    if args.hf is None:
        raise SystemExit("--hf_bucket is required")
    if args.sharded is None and not (args.already_downloaded or args.already_unsharded):
        raise SystemExit("--sharded_bucket is required unless the checkpoint is already local (--already_downloaded / --already_unsharded)")

    from storage_cleaner import copy_tree
    from unshard import main as unshard

    from olmo_b200.config import ShardedCheckpointerType, TrainConfig
    from olmo_b200.hf.convert import write_hf_olmo_checkpoint, write_transformers_checkpoint

    work = Path(args.local_dir) if args.local_dir else Path(tempfile.mkdtemp(prefix="unshard_to_hf_"))
    work.mkdir(parents=True, exist_ok=True)
    sharded, unsharded, hf = work / "sharded", work / "unsharded", work / "hf"

    if not args.already_unsharded:
        if not args.already_downloaded:
            log.info("fetching %s", args.sharded)
            copy_tree(args.sharded, str(sharded), dry_run=False)
        cfg = TrainConfig.load(sharded / "config.yaml", validate_paths=False)
        kind = ShardedCheckpointerType(args.type) if args.type else cfg.sharded_checkpointer
        log.info("unsharding into %s", unsharded)
        unshard(sharded, unsharded, sharded_checkpoint_type=kind, model_only=args.model_only)
        if args.unsharded:
            copy_tree(str(unsharded), args.unsharded, dry_run=False)
    elif not (unsharded / "config.yaml").is_file():
        if args.unsharded is None:
            raise SystemExit(f"--already_unsharded: neither {unsharded} nor --unsharded_bucket holds the checkpoint")
        copy_tree(args.unsharded, str(unsharded), dry_run=False)

    style = "hf_olmo" if args.hf_olmo else args.style
    log.info("converting to the %s layout", style)
    if style == "transformers":
        write_transformers_checkpoint(unsharded, hf, tokenizer_path=args.tokenizer)
    else:
        write_hf_olmo_checkpoint(unsharded, hf, tokenizer_path=args.tokenizer)
    copy_tree(str(hf), args.hf, dry_run=False)
    if args.cleanup_local_dir:
        shutil.rmtree(work, ignore_errors=True)
    print(args.hf)
    return args.hf


if __name__ == "__main__":
    main()
