#!/usr/bin/env python
"""Unsharded OLMo-2 checkpoint -> ``transformers`` ``Olmo2ForCausalLM`` directory (reference: ``scripts/convert_olmo2_to_hf.py``).

    python scripts/convert_olmo2_to_hf.py --input_dir CKPT --output_dir OUT [--tokenizer_json_path tok.json] [--dtype bfloat16]
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
    args = ap.parse_args()
    out, model_type = write_transformers_checkpoint(
        args.input_dir, args.output_dir, tokenizer_path=args.tokenizer_json_path, dtype=getattr(torch, args.dtype) if args.dtype else None
    )
    if model_type != expect:
        print(f"warning: the checkpoint's architecture maps to '{model_type}', not '{expect}'", file=sys.stderr)
    print(out)


if __name__ == "__main__":
    main()
