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
    """Greedy continuation of text prompts with a KV cache; prompts of one request are batched with left padding.
    ``stop_sequences`` cut a continuation at the first occurrence of any of the strings (the role of the stop-id criterion in
    the reference's ``generate_completions``, ``inference/eval/utils.py:17-107``)."""

    def __init__(self, model, tokenizer, max_new_tokens: int = 256, device: Optional[torch.device] = None,
                 stop_sequences: Optional[List[str]] = None):
        self.model, self.tokenizer, self.max_new_tokens = model.eval(), tokenizer, max_new_tokens
        self.device = device or next(model.parameters()).device
        self.stop_sequences = list(stop_sequences or [])

    def _left_padded(self, inputs: List[str]):
        encoded = [self.tokenizer.encode(text, add_special_tokens=False) or [self.tokenizer.eos_token_id] for text in inputs]
        width = min(max(len(e) for e in encoded), self.model.config.max_sequence_length)
        ids = torch.full((len(encoded), width), self.tokenizer.pad_token_id, dtype=torch.long)
        mask = torch.zeros(len(encoded), width)
        for i, e in enumerate(encoded):
            e = e[-width:]
            ids[i, width - len(e) :] = torch.tensor(e)
            mask[i, width - len(e) :] = 1
        return ids.to(self.device), mask.to(self.device), width

    @torch.no_grad()
    def predict(self, inputs: List[str]) -> Iterator[str]:
        ids, mask, width = self._left_padded(inputs)
        room = self.model.config.max_sequence_length - width
        out = self.model.generate(ids, attention_mask=mask, max_steps=max(1, min(self.max_new_tokens, room)), beam_size=1)
        for row in out.token_ids[:, 0].tolist():
            if self.tokenizer.eos_token_id in row:
                row = row[: row.index(self.tokenizer.eos_token_id)]
            text = self.tokenizer.decode(row)
            cuts = [text.index(s) for s in self.stop_sequences if s and s in text]
            if cuts:
                text = text[: min(cuts)]
            yield text.strip()

    @torch.no_grad()
    def next_token_predictions(self, inputs: List[str], candidate_token_ids: Optional[List[int]] = None, batch_size: int = 8):
        """For every prompt: the index of the most likely next token among ``candidate_token_ids`` (or in the whole
        vocabulary) and the probabilities over those candidates (``get_next_word_predictions``,
        ``inference/eval/utils.py:110-155``)."""
        picks: List[int] = []
        probs: List[List[float]] = []
        for start in range(0, len(inputs), batch_size):
            ids, mask, _ = self._left_padded(inputs[start : start + batch_size])
            logits = self.model(ids, attention_mask=mask, last_logits_only=True).logits[:, -1].float()
            p = torch.softmax(logits, dim=-1)
            if candidate_token_ids is not None:
                p = p[:, candidate_token_ids]
            picks += p.argmax(dim=-1).tolist()
            probs += p.tolist()
        return picks, probs


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
