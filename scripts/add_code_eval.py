#!/usr/bin/env python
"""
Turn code datasets into perplexity evaluation files: one ``{"id", "text", "metadata"}`` object per line, gzipped, where
``text`` is the prompt followed by its reference solution (the role of the reference's ``scripts/add_code_eval.py``).
The outputs are inputs of the offline pipeline's ``ppl`` task (``evaluation/``).

    python scripts/add_code_eval.py OUTDIR                         # HumanEval test, MBPP validation and test
    python scripts/add_code_eval.py OUTDIR --dataset PATH --split test --id-key id --prompt-key question --answer-key answer

Datasets are read from disk first (``OLMO_DATA_DIR/hf_datasets/<path>/<name>/<split>`` as written by
``datasets.save_to_disk``) and from the hub otherwise.
"""
import argparse
import gzip
import json
import sys
from pathlib import Path
from typing import Any, Dict, Iterable, Optional

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

PRESETS = [
    # (dataset path, config name, split, id key, prompt key, answer key, output file)
    ("openai_humaneval", None, "test", "task_id", "prompt", "canonical_solution", "openai_humaneval_test.jsonl.gz"),
    ("mbpp", None, "validation", "task_id", "text", "code", "mbpp_validation.jsonl.gz"),
    ("mbpp", None, "test", "task_id", "text", "code", "mbpp_test.jsonl.gz"),
]


def load_split(path: str, name: Optional[str], split: str) -> Iterable[Dict[str, Any]]:
    try:
        from olmo_b200.eval.downstream import load_hf_dataset

        return load_hf_dataset(path, name, split)
    except FileNotFoundError:
        import datasets

        return datasets.load_dataset(path, name, split=split)


def write_raw_dataset(rows: Iterable[Dict[str, Any]], id_key: str, prompt_key: str, answer_key: str, save_to: Path) -> int:
    save_to.parent.mkdir(parents=True, exist_ok=True)
    n = 0
    with gzip.open(save_to, "wt", encoding="utf-8") as f:
        for row in rows:
            row = dict(row)
            record = {"id": row.pop(id_key), "text": row.pop(prompt_key) + row.pop(answer_key), "metadata": row}
            f.write(json.dumps(record, default=str) + "\n")
            n += 1
    return n


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("outdir")
    ap.add_argument("--dataset", default=None, help="a dataset path instead of the presets")
    ap.add_argument("--name", default=None)
    ap.add_argument("--split", default="test")
    ap.add_argument("--id-key", default="task_id")
    ap.add_argument("--prompt-key", default="prompt")
    ap.add_argument("--answer-key", default="canonical_solution")
    args = ap.parse_args(argv)
    out = Path(args.outdir)
    jobs = PRESETS if args.dataset is None else [
        (args.dataset, args.name, args.split, args.id_key, args.prompt_key, args.answer_key, f"{Path(args.dataset).name}_{args.split}.jsonl.gz")]
    for path, name, split, id_key, prompt_key, answer_key, file in jobs:
        n = write_raw_dataset(load_split(path, name, split), id_key, prompt_key, answer_key, out / file)
        print(f"{out / file}: {n} documents")
    return 0


if __name__ == "__main__":
    sys.exit(main())
