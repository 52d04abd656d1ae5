#!/usr/bin/env python
"""OLMo checkpoint -> ``hf_olmo`` layout (``config.json``, ``model.safetensors`` with ``model.`` key prefix, tokenizer files);
sharded checkpoints are unsharded first (reference: ``hf_olmo/convert_olmo_to_hf.py:34-316``).

    python hf_olmo/convert_olmo_to_hf.py --checkpoint-dir CKPT [--destination-dir OUT] [--tokenizer tok.json] [--keep-olmo-artifacts]
"""
import argparse
import sys
import tempfile
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--checkpoint-dir", required=True)
    ap.add_argument("--destination-dir", default=None)
    ap.add_argument("--tokenizer", default=None, help="tokenizer.json to ship instead of the one named in config.yaml")
    ap.add_argument("--keep-olmo-artifacts", action="store_true")
    ap.add_argument("--pytorch-bin", action="store_true", help="write pytorch_model.bin instead of safetensors")
    args = ap.parse_args()

    from olmo_b200.hf.convert import write_hf_olmo_checkpoint

    src = Path(args.checkpoint_dir)
    if not ((src / "model.pt").is_file() or (src / "model.safetensors").is_file()):
        # a sharded checkpoint: gather it on the host first
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "scripts"))
        from unshard import main as unshard
        from olmo_b200.config import TrainConfig

        cfg = TrainConfig.load(src / "config.yaml", validate_paths=False)
        tmp = Path(tempfile.mkdtemp(prefix="unsharded_"))
        unshard(src, tmp, sharded_checkpoint_type=cfg.sharded_checkpointer, model_only=True)
        src = tmp
    out = write_hf_olmo_checkpoint(
        src, args.destination_dir or args.checkpoint_dir, tokenizer_path=args.tokenizer, safe_serialization=not args.pytorch_bin,
        keep_olmo_artifacts=args.keep_olmo_artifacts or args.destination_dir is not None,
    )
    print(out)


if __name__ == "__main__":
    main()
