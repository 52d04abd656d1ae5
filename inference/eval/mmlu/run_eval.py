#!/usr/bin/env python
"""MMLU accuracy of a local checkpoint (full precision or 4-bit) or of a served model.

    python inference/eval/mmlu/run_eval.py --model_name_or_path CKPT [--gptq] [--ntrain 5] [--subjects s1 s2 ...]
        [--n_instances N] [--eval_batch_size B] [--save_dir OUT]
    python inference/eval/mmlu/run_eval.py --openai_engine MODEL --base_url http://host:8000/v1 [--use_chat_format] ...

The options are those of the reference's script of this path; ``--openai_engine`` evaluates any OpenAI-compatible endpoint
(``--base_url``, default ``OPENAI_BASE_URL`` or the public API) through :mod:`olmo_b200.inference.remote`.  Questions come
from the packaged MMLU files (``olmo_data/hf_datasets/hails/mmlu_no_train``), so ``--data_dir`` is accepted and unused.
``--save_dir`` receives ``metrics.json``.
"""
import argparse
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[3]))


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ntrain", type=int, default=5)
    ap.add_argument("--data_dir", default=None, help="accepted for compatibility")
    ap.add_argument("--save_dir", default=None)
    ap.add_argument("--model_name_or_path", default=None, help="checkpoint folder (or quantised folder with --gptq)")
    ap.add_argument("--tokenizer_name_or_path", default=None)
    ap.add_argument("--openai_engine", default=None, help="model name at an OpenAI-compatible endpoint")
    ap.add_argument("--base_url", default=os.environ.get("OPENAI_BASE_URL", "https://api.openai.com/v1"))
    ap.add_argument("--subjects", nargs="*", default=None, help="subjects, fields or groups (default: all four groups)")
    ap.add_argument("--n_instances", type=int, default=None, help="at most this many questions per evaluated group")
    ap.add_argument("--eval_batch_size", type=int, default=1)
    ap.add_argument("--load_in_8bit", action="store_true", help="accepted for compatibility (weights are bf16 or 4-bit here)")
    ap.add_argument("--gptq", action="store_true", help="--model_name_or_path is a folder written by run_quantization.py")
    ap.add_argument("--use_chat_format", action="store_true")
    args = ap.parse_args(argv)
    if (args.model_name_or_path is None) == (args.openai_engine is None):
        ap.error("give exactly one of --model_name_or_path and --openai_engine")
    groups = args.subjects or ["stem", "humanities", "social_sciences", "other"]
    results = {}
    if args.openai_engine is not None:
        from olmo_b200.inference.remote import score_mmlu_remote
        from olmo_b200.tokenizer import Tokenizer

        ident = args.tokenizer_name_or_path or "tokenizers/allenai_dolma2.json"
        tokenizer = Tokenizer.from_file(ident) if os.path.exists(ident) else Tokenizer.from_pretrained(ident)
        for group in groups:
            cache = str(Path(args.save_dir) / f"{group}.jsonl") if args.save_dir else None
            results[group] = score_mmlu_remote(args.base_url, args.openai_engine, tokenizer, group=group, shots=args.ntrain, limit=args.n_instances,
                                               chat=args.use_chat_format, output_path=cache, api_key=os.environ.get("OPENAI_API_KEY"),
                                               batch_size=max(args.eval_batch_size, 1))
    else:
        import torch

        from olmo_b200.inference.efficiency import load_quantized
        from olmo_b200.inference.mmlu_eval import score_mmlu
        from olmo_b200.models.olmo import OLMo
        from olmo_b200.tokenizer import Tokenizer

        device = "cuda" if torch.cuda.is_available() else "cpu"
        model = load_quantized(args.model_name_or_path, device) if args.gptq else OLMo.from_checkpoint(args.model_name_or_path, device=device)
        tokenizer = Tokenizer.from_file(args.tokenizer_name_or_path) if args.tokenizer_name_or_path else Tokenizer.from_checkpoint(args.model_name_or_path)
        for group in groups:
            results[group] = score_mmlu(model, tokenizer, group, "test", args.ntrain, args.eval_batch_size, args.n_instances)
    total = sum(r["n"] for r in results.values()) or 1.0
    results["average_acc"] = sum(r["acc"] * r["n"] for r in results.values() if isinstance(r, dict)) / total
    print(json.dumps(results, indent=2))
    if args.save_dir:
        Path(args.save_dir).mkdir(parents=True, exist_ok=True)
        (Path(args.save_dir) / "metrics.json").write_text(json.dumps(results, indent=2))
    return results


if __name__ == "__main__":
    main()
