#!/usr/bin/env python
"""Chat-format SFT data -> ``input_ids.npy`` (uint16/uint32) + ``label_mask.npy`` (bool), one fixed-length instance per
conversation: ``<eos>`` then ``<|role|>\\n content\\n`` per message; only assistant contents (and their closing EOS) are
trained on (reference: ``scripts/prepare_tulu_data.py``).  Conversations come from a JSON-lines file of
``{"messages": [{"role":..., "content":...}, ...]}`` records or from a ``datasets`` dataset on disk / the Hub.

    python scripts/prepare_tulu_data.py OUT_DIR --source conversations.jsonl -t tokenizer.json -s 2048 --eos 50279 --pad 1
"""
from __future__ import annotations

import argparse
import json
import logging
import sys
from pathlib import Path
from typing import Dict, Iterable, List

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np

log = logging.getLogger("prepare_tulu_data")


def render(messages: List[Dict[str, str]], tokenizer, max_seq_len: int) -> Dict[str, list]:
    ids, mask = [tokenizer.eos_token_id], [False]
    for msg in messages:
        role = tokenizer.encode(f"<|{msg['role']}|>\n", add_special_tokens=False)
        ids += role
        mask += [False] * len(role)
        if msg["role"] == "assistant":
            content = tokenizer.encode(msg["content"].strip() + tokenizer.eos_token + "\n", add_special_tokens=False)
            mask += [True] * len(content)
            if len(content) >= 2 and content[-2] == tokenizer.eos_token_id:
                mask[-1] = False  # the newline after EOS is not a target
        else:
            content = tokenizer.encode(msg["content"].strip() + "\n", add_special_tokens=False)
            mask += [False] * len(content)
        ids += content
    ids, mask = ids[:max_seq_len], mask[:max_seq_len]
    pad = max_seq_len - len(ids)
    return {"input_ids": ids + [tokenizer.pad_token_id] * pad, "label_mask": mask + [False] * pad, "n_labels": sum(mask)}


def conversations(source: str) -> Iterable[List[Dict[str, str]]]:
    p = Path(source)
    if p.is_file():
        with open(p) as f:
            for line in f:
                if line.strip():
                    yield json.loads(line)["messages"]
        return
    import datasets

    ds = datasets.load_from_disk(source) if p.is_dir() else datasets.load_dataset(source, split="train")
    for ex in ds:
        yield ex["messages"]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("output_dir")
    ap.add_argument("--source", default="allenai/tulu-v2-sft-mixture")
    ap.add_argument("-t", "--tokenizer", required=True)
    ap.add_argument("-s", "--seq-len", type=int, default=2048)
    ap.add_argument("--eos", type=int, default=50279)
    ap.add_argument("--pad", type=int, default=1)
    ap.add_argument("-j", "--num-proc", type=int, default=1, help="worker threads that render and tokenise conversations")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO)
    from olmo_b200.tokenizer import Tokenizer

    kwargs = dict(eos_token_id=args.eos, pad_token_id=args.pad)
    tok = Tokenizer.from_file(args.tokenizer, **kwargs) if Path(args.tokenizer).is_file() else Tokenizer.from_pretrained(args.tokenizer, **kwargs)
    if args.num_proc > 1:  # the tokenizer library releases the interpreter lock while it encodes
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(max_workers=args.num_proc) as pool:
            rows = list(pool.map(lambda m: render(m, tok, args.seq_len), conversations(args.source)))
    else:
        rows = [render(m, tok, args.seq_len) for m in conversations(args.source)]
    kept = [r for r in rows if r["n_labels"] > 0]
    log.info("kept %d of %d conversations", len(kept), len(rows))
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    total = len(kept) * args.seq_len
    dtype = np.uint16 if tok.vocab_size <= 65536 else np.uint32
    ids = np.memmap(out / "input_ids.npy", dtype=dtype, mode="w+", shape=(max(total, 1),))
    mask = np.memmap(out / "label_mask.npy", dtype=np.bool_, mode="w+", shape=(max(total, 1),))
    for i, r in enumerate(kept):
        ids[i * args.seq_len : (i + 1) * args.seq_len] = r["input_ids"]
        mask[i * args.seq_len : (i + 1) * args.seq_len] = r["label_mask"]
    ids.flush()
    mask.flush()
    log.info("wrote %s tokens to %s", f"{total:,}", out)
    return len(kept)


if __name__ == "__main__":
    main()
