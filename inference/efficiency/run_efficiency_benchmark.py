#!/usr/bin/env python
"""Predictor for an efficiency-benchmark harness: reads JSON lists of prompts on stdin, writes JSON lists of continuations on
stdout, one line each (the protocol of the reference's script of this name).

    python inference/efficiency/run_efficiency_benchmark.py --pretrained-model-dir CKPT [--quantized-model-dir QDIR] [--vllm]

``--vllm`` selects the framework's continuous-batching engine (:mod:`olmo_b200.serve`) instead of the plain predictor; the
third-party server of that name is not used.
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


class EnginePredictor:
    """The serving engine behind the predictor interface (``predict(list of prompts) -> iterator of continuations``)."""

    def __init__(self, checkpoint_dir: str, max_new_tokens: int = 256):
        import torch

        from olmo_b200.serve import SamplingParams, load_engine

        device = "cuda" if torch.cuda.is_available() else "cpu"
        self.engine = load_engine(checkpoint_dir, device=device, dtype="bf16" if device == "cuda" else "fp32")
        self.params = SamplingParams(max_tokens=max_new_tokens, temperature=0.0)

    def predict(self, inputs):
        prompts = [self.engine.tokenizer.encode(text, add_special_tokens=False) or [self.engine.tokenizer.eos_token_id] for text in inputs]
        for done in self.engine.generate(prompts, self.params):
            yield done.text.strip()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--pretrained-model-dir", required=True)
    ap.add_argument("--quantized-model-dir", default=None, nargs="?")
    ap.add_argument("--vllm", action="store_true", help="use the continuous-batching engine")
    ap.add_argument("--max-new-tokens", type=int, default=256)
    args = ap.parse_args(argv)
    from olmo_b200.inference.efficiency import Predictor, load_quantized, stdio_predictor_wrapper

    if args.vllm:
        predictor = EnginePredictor(args.pretrained_model_dir, args.max_new_tokens)
    else:
        import torch

        from olmo_b200.models.olmo import OLMo
        from olmo_b200.tokenizer import Tokenizer

        device = "cuda" if torch.cuda.is_available() else "cpu"
        model = load_quantized(args.quantized_model_dir, device) if args.quantized_model_dir else OLMo.from_checkpoint(args.pretrained_model_dir, device=device)
        predictor = Predictor(model, Tokenizer.from_checkpoint(args.quantized_model_dir or args.pretrained_model_dir), max_new_tokens=args.max_new_tokens)
    return stdio_predictor_wrapper(predictor, sys.stdin, sys.stdout)


if __name__ == "__main__":
    main()
