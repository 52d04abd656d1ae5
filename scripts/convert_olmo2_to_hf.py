#!/usr/bin/env python
"""Unsharded OLMo-2 checkpoint -> ``transformers`` ``Olmo2ForCausalLM`` directory (reference: ``scripts/convert_olmo2_to_hf.py``).

    python scripts/convert_olmo2_to_hf.py --input_dir CKPT --output_dir OUT [--tokenizer_json_path tok.json] [--dtype bfloat16]
                                          [--no_tokenizer] [--no_fix_eos_token_id] [--no_safe_serialization]
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch

from olmo_b200.hf.convert import write_transformers_checkpoint


def main(expect: str = "olmo2") -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--input_dir", required=True, help="unsharded checkpoint directory (config.yaml + model.pt/.safetensors)")
    ap.add_argument("--output_dir", required=True)
    ap.add_argument("--tokenizer_json_path", default=None)
    ap.add_argument("--dtype", default=None, choices=[None, "float32", "bfloat16", "float16"])
    ap.add_argument("--no_tokenizer", action="store_false", dest="include_tokenizer", help="write no tokenizer files")
    ap.add_argument("--no_fix_eos_token_id", action="store_false", dest="fix_eos_token_id",
                    help="keep an end-of-text id of 0 instead of exporting 50279 for it (the correction is a bug fix: use with care)")
    ap.add_argument("--no_safe_serialization", action="store_false", dest="safe_serialization", help="write pytorch_model.bin instead of safetensors")
    ap.add_argument("--safe_serialization", action="store_true", dest="safe_serialization", help="write safetensors (the default)")
    ap.add_argument("--no_tmp_cleanup", action="store_true", help="accepted for compatibility: this converter writes no temporary folder")
    ap.set_defaults(safe_serialization=True)
    args = ap.parse_args()
    out, model_type = write_transformers_checkpoint(
        args.input_dir, args.output_dir, tokenizer_path=args.tokenizer_json_path, dtype=getattr(torch, args.dtype) if args.dtype else None,
        include_tokenizer=args.include_tokenizer, safe_serialization=args.safe_serialization, fix_eos_token_id=args.fix_eos_token_id,
    )
    if model_type != expect:
        print(f"warning: the checkpoint's architecture maps to '{model_type}', not '{expect}'", file=sys.stderr)
    print(out)


if __name__ == "__main__":
    main()
