#!/usr/bin/env python
"""List what an experiment's task sets may name: the shipped task-set files and every task label
(reference counterpart: ``evaluation/see_available_tasks.py``)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> int:
    from olmo_b200.eval.downstream import label_to_task_map
    from olmo_b200.eval.offline import TASK_SET_DIR

    print("task sets:")
    for file in sorted(TASK_SET_DIR.glob("*.yaml")):
        print(f"  {file.stem}")
    print("tasks:")
    print("  ppl  (task_kwargs: files=[...jsonl(.gz) | ...npy], text_field, memmap_dtype)")
    for label in sorted(label_to_task_map):
        print(f"  {label}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
