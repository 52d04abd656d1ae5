"""
MMLU scoring of a checkpoint (full precision or quantised) outside the training loop: k-shot prompts with lettered
choices, the answer is the letter with the highest next-token probability.  Same protocol as the reference's
``inference/eval/mmlu/run_eval.py`` (which follows the original MMLU script); prompt construction is shared with the
in-loop task :class:`olmo_b200.eval.downstream.MMLU`.

    python -m olmo_b200.inference.mmlu_eval --checkpoint-dir CKPT [--quantized-model-dir Q] [--group stem] [--ntrain 5] [--split test]
"""
from __future__ import annotations

import argparse
import json
from collections import defaultdict
from typing import Dict, List, Optional

import torch

__all__ = ["score_mmlu"]


@torch.no_grad()
def score_mmlu(model, tokenizer, group: str = "stem", split: str = "test", shots: int = 5, batch_size: int = 4, limit: Optional[int] = None,
               device: Optional[torch.device] = None) -> Dict[str, float]:
    """Accuracy per subject and overall; reads the MMLU files from the packaged-data tree (``hf_datasets/hails/mmlu_no_train``)."""
    from ..eval.downstream import MMLU

    task = MMLU(tokenizer, dataset_name=group, split=split, prompt_variations=2 if shots > 0 else None, mc_labels=True)
    device = device or next(model.parameters()).device
    letter_ids = [tokenizer.encode(f" {c}", add_special_tokens=False)[-1] for c in "ABCD"]
    # one request per document is enough: all four continuations share the context and differ in the final letter
    docs: Dict[int, Dict] = {}
    for s in task.samples:
        docs.setdefault(s["doc_id"], s)
    rows = list(docs.values())[:limit]
    subjects = [d.get("subject", "all") for d in task.dataset][: len(rows)] if hasattr(task.dataset, "__iter__") else ["all"] * len(rows)
    hits: Dict[str, List[int]] = defaultdict(list)
    model.eval()
    for start in range(0, len(rows), batch_size):
        chunk = rows[start : start + batch_size]
        width = max(len(r["ctx"]) for r in chunk)
        width = min(width, model.config.max_sequence_length)
        ids = torch.full((len(chunk), width), tokenizer.pad_token_id, dtype=torch.long)
        mask = torch.zeros(len(chunk), width)
        for i, r in enumerate(chunk):
            ctx = r["ctx"][-width:]
            ids[i, width - len(ctx) :] = torch.tensor(ctx)
            mask[i, width - len(ctx) :] = 1
        logits = model(ids.to(device), attention_mask=mask.to(device), last_logits_only=True).logits[:, -1]
        pred = logits[:, letter_ids].argmax(dim=-1).tolist()
        for i, r in enumerate(chunk):
            ok = int(pred[i] == r["label_id"])
            hits[subjects[start + i] if start + i < len(subjects) else "all"].append(ok)
            hits["__all__"].append(ok)
    out = {f"acc/{k}": sum(v) / len(v) for k, v in hits.items() if k != "__all__"}
    out["acc"] = sum(hits["__all__"]) / max(1, len(hits["__all__"]))
    out["n"] = float(len(hits["__all__"]))
    return out


def main(argv=None) -> Dict[str, float]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--checkpoint-dir", default=None)
    ap.add_argument("--quantized-model-dir", default=None)
    ap.add_argument("--group", default="stem", help="stem | humanities | social_sciences | other | a field | a subject")
    ap.add_argument("--split", default="test")
    ap.add_argument("--ntrain", type=int, default=5)
    ap.add_argument("--batch-size", type=int, default=4)
    ap.add_argument("--limit", type=int, default=None)
    args = ap.parse_args(argv)
    from ..models.olmo import OLMo
    from ..tokenizer import Tokenizer
    from .efficiency import load_quantized

    device = "cuda" if torch.cuda.is_available() else "cpu"
    folder = args.quantized_model_dir or args.checkpoint_dir
    model = load_quantized(folder, device) if args.quantized_model_dir else OLMo.from_checkpoint(folder, device=device)
    result = score_mmlu(model, Tokenizer.from_checkpoint(folder), args.group, args.split, args.ntrain, args.batch_size, args.limit)
    print(json.dumps(result, indent=2))
    return result


if __name__ == "__main__":
    main()
