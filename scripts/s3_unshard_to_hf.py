#!/usr/bin/env python
"""Remote sharded checkpoint -> local copy -> unsharded -> HuggingFace directory -> upload (reference:
``scripts/s3_unshard_to_hf.py``).  Works with every storage scheme the framework addresses (s3, r2, weka, gs, local).

    python scripts/s3_unshard_to_hf.py --sharded-url s3://bucket/run/step1000 --hf-url s3://bucket/run/step1000-hf \\
        [--unsharded-url s3://bucket/run/step1000-unsharded] [--layout transformers|hf_olmo] [--tmp-dir /scratch]
"""
import argparse
import sys
import tempfile
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--sharded-url", required=True)
    ap.add_argument("--hf-url", required=True)
    ap.add_argument("--unsharded-url", default=None, help="also keep the unsharded checkpoint here")
    ap.add_argument("--layout", choices=["transformers", "hf_olmo"], default="transformers")
    ap.add_argument("--tmp-dir", default=None)
    ap.add_argument("--tokenizer", default=None)
    args = ap.parse_args(argv)

    from storage_cleaner import copy_tree
    from unshard import main as unshard

    from olmo_b200.config import TrainConfig
    from olmo_b200.hf.convert import write_hf_olmo_checkpoint, write_transformers_checkpoint

    work = Path(tempfile.mkdtemp(prefix="unshard_to_hf_", dir=args.tmp_dir))
    sharded, unsharded, hf = work / "sharded", work / "unsharded", work / "hf"
    copy_tree(args.sharded_url, str(sharded), dry_run=False)
    cfg = TrainConfig.load(sharded / "config.yaml", validate_paths=False)
    unshard(sharded, unsharded, sharded_checkpoint_type=cfg.sharded_checkpointer, model_only=True)
    if args.unsharded_url:
        copy_tree(str(unsharded), args.unsharded_url, dry_run=False)
    if args.layout == "transformers":
        write_transformers_checkpoint(unsharded, hf, tokenizer_path=args.tokenizer)
    else:
        write_hf_olmo_checkpoint(unsharded, hf, tokenizer_path=args.tokenizer)
    copy_tree(str(hf), args.hf_url, dry_run=False)
    print(args.hf_url)


if __name__ == "__main__":
    main()
