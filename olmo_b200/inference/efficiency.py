"""
Efficiency-benchmark predictor: a loop that reads one JSON list of prompts per line from stdin and writes one JSON list
of completions per line to stdout, which is the protocol of the efficiency-pentathlon harness the reference targets
(``inference/efficiency/run_efficiency_benchmark.py:16-114``).  The model is a native OLMo checkpoint, optionally
quantised to 4 bit on load (``--quantize rtn``) or loaded from a directory written by ``run_quantization`` below.

    python -m olmo_b200.inference.efficiency --checkpoint-dir CKPT [--quantize rtn] [--max-new-tokens 256] < prompts.jsonl
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Iterable, Iterator, List, Optional, TextIO

import torch

__all__ = ["Predictor", "stdio_predictor_wrapper", "run_quantization", "load_quantized"]


class Predictor:
    """Greedy continuation of text prompts with a KV cache; prompts of one request are batched with left padding."""

    def __init__(self, model, tokenizer, max_new_tokens: int = 256, device: Optional[torch.device] = None):
        self.model, self.tokenizer, self.max_new_tokens = model.eval(), tokenizer, max_new_tokens
        self.device = device or next(model.parameters()).device

    @torch.no_grad()
    def predict(self, inputs: List[str]) -> Iterator[str]:
        encoded = [self.tokenizer.encode(text, add_special_tokens=False) or [self.tokenizer.eos_token_id] for text in inputs]
        width = max(len(e) for e in encoded)
        ids = torch.full((len(encoded), width), self.tokenizer.pad_token_id, dtype=torch.long)
        mask = torch.zeros(len(encoded), width)
        for i, e in enumerate(encoded):
            ids[i, width - len(e) :] = torch.tensor(e)
            mask[i, width - len(e) :] = 1
        room = self.model.config.max_sequence_length - width
        out = self.model.generate(ids.to(self.device), attention_mask=mask.to(self.device), max_steps=max(1, min(self.max_new_tokens, room)), beam_size=1)
        for row in out.token_ids[:, 0].tolist():
            if self.tokenizer.eos_token_id in row:
                row = row[: row.index(self.tokenizer.eos_token_id)]
            yield self.tokenizer.decode(row).strip()


def stdio_predictor_wrapper(predictor: Predictor, stdin: TextIO = sys.stdin, stdout: TextIO = sys.stdout) -> int:
    served = 0
    for line in stdin:
        line = line.rstrip()
        if not line:
            continue
        batch = json.loads(line)
        assert isinstance(batch, list)
        stdout.write(json.dumps(list(predictor.predict(batch))) + "\n")
        stdout.flush()  # the harness reads through a pipe and waits for each answer
        served += 1
    return served


def run_quantization(checkpoint_dir: str, output_dir: str, calibration: Iterable[torch.Tensor], *, group: int = 128, act_order: bool = True,
                     method: str = "gptq", device: str = "cpu") -> Path:
    """Quantise an unsharded checkpoint and store ``config.yaml`` + ``quantized.pt`` (packed buffers + remaining weights)."""
    from ..models.olmo import OLMo
    from .quantize import quantize_model

    model = OLMo.from_checkpoint(checkpoint_dir, device=device)
    report = quantize_model(model, list(calibration), group=group, act_order=act_order, method=method)
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    (out / "config.yaml").write_text((Path(checkpoint_dir) / "config.yaml").read_text())
    torch.save({"state": model.state_dict(), "group": group, "act_order": act_order and method == "gptq", "report": report}, out / "quantized.pt")
    return out


def load_quantized(quantized_dir: str, device: str = "cpu"):
    """Rebuild the model skeleton, swap the block linears for :class:`QuantLinear` and load the packed buffers."""
    from ..config import ModelConfig
    from ..models.olmo import OLMo
    from .quantize import BLOCK_LINEARS
    from .w4a16 import QuantLinear

    folder = Path(quantized_dir)
    blob = torch.load(folder / "quantized.pt", map_location="cpu", weights_only=False)
    cfg = ModelConfig.load(folder / "config.yaml", key="model", validate_paths=False)
    cfg.init_device = "cpu"
    model = OLMo(cfg, init_params=False)
    for block in model.all_blocks():
        block._fused_ok = False  # packed weights: module path only
        for name in BLOCK_LINEARS:
            old = getattr(block, name, None)
            if isinstance(old, torch.nn.Linear):
                setattr(block, name, QuantLinear(old.in_features, old.out_features, group=blob["group"], bias=old.bias is not None, act_order=blob["act_order"]))
    model.load_state_dict(blob["state"])
    return model.to(device).eval()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--checkpoint-dir", "--pretrained-model-dir", dest="checkpoint_dir", default=None)
    ap.add_argument("--quantized-model-dir", default=None)
    ap.add_argument("--quantize", choices=["none", "rtn"], default="none", help="quantise on load without calibration data")
    ap.add_argument("--max-new-tokens", type=int, default=256)
    args = ap.parse_args(argv)
    from ..models.olmo import OLMo
    from ..tokenizer import Tokenizer

    device = "cuda" if torch.cuda.is_available() else "cpu"
    if args.quantized_model_dir:
        model = load_quantized(args.quantized_model_dir, device)
        tokenizer = Tokenizer.from_checkpoint(args.quantized_model_dir)
    else:
        model = OLMo.from_checkpoint(args.checkpoint_dir, device=device)
        tokenizer = Tokenizer.from_checkpoint(args.checkpoint_dir)
        if args.quantize == "rtn":
            from .quantize import quantize_model

            quantize_model(model, [torch.full((1, 8), tokenizer.eos_token_id)], method="rtn")
    return stdio_predictor_wrapper(Predictor(model, tokenizer, args.max_new_tokens))


if __name__ == "__main__":
    main()
