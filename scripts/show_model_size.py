#!/usr/bin/env python
"""Parameter counts of the model a training config describes, where they sit, and what training it needs per GPU.

    scripts/show_model_size.py CONFIG.yaml [--model.key=value ...]

The two totals (all parameters; without the embedding) are what the reference's ``scripts/show_model_size.py`` logs.  Below
them: the share of the embedding, one block and the output head, and the device memory the flat-shard engine holds per GPU
for 1 to 8 GPUs under both schedules (fp32 master, gradient and two AdamW moments are sharded: 16 bytes per parameter
over the ranks; the resident schedule adds a gathered bf16 copy and an fp32 gradient accumulator: 6 bytes per parameter
on every rank; the sharded schedule keeps those only for the embedding, the head and five block-sized slots).
"""
import logging
import sys
from pathlib import Path
from typing import Dict

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.config import TrainConfig
from olmo_b200.exceptions import OLMoCliError
from olmo_b200.models.olmo import OLMo
from olmo_b200.util import clean_opt, prepare_cli_environment

log = logging.getLogger(__name__)


def count(cfg: TrainConfig) -> Dict[str, int]:
    """Counts from a one-block copy of the model on the meta device (no storage is allocated)."""
    model_cfg = cfg.model
    layers, model_cfg.n_layers, model_cfg.init_device = model_cfg.n_layers, 1, "meta"
    try:
        probe = OLMo(model_cfg, init_params=False)
    finally:
        model_cfg.n_layers = layers
    block = sum(p.numel() for p in probe.transformer.blocks.parameters())  # type: ignore[union-attr]
    with_one = probe.num_params()
    embedding = with_one - probe.num_params(include_embedding=False)
    head = sum(p.numel() for n, p in probe.named_parameters() if n.startswith("transformer.ff_out"))
    total = with_one + block * (layers - 1)
    return {"total": total, "non_embedding": total - embedding, "embedding": embedding, "block": block, "blocks": layers, "head": head,
            "other": total - embedding - head - block * layers}


def memory_plan(sizes: Dict[str, int], gpus: int) -> Dict[str, float]:
    """GB of engine state per GPU (activations and workspaces come on top)."""
    p, block = sizes["total"], sizes["block"]
    if gpus == 1:  # nothing is gathered: master, gradient and two moments in fp32 plus the bf16 copy the GEMMs read
        return {"resident": 18 * p / 1e9, "sharded": 18 * p / 1e9}
    shards = 16 * p / gpus
    resident = shards + 6 * p
    outside = p - block * sizes["blocks"]  # embedding, head, final norm: gathered in both schedules
    sharded = shards + 6 * outside + (2 * 2 + 3 * 4) * block  # two bf16 parameter slots, three fp32 gradient slots
    return {"resident": resident / 1e9, "sharded": sharded / 1e9}


def main(cfg: TrainConfig) -> Dict[str, int]:
    sizes = count(cfg)
    log.info("Total number of parameters: %s", f"{sizes['total']:,d}")
    log.info("Number of non-embedding parameters: %s", f"{sizes['non_embedding']:,d}")
    for name in ("embedding", "head", "other"):
        log.info("  %-12s %16s  (%4.1f %%)", name, f"{sizes[name]:,d}", 100 * sizes[name] / sizes["total"])
    log.info("  %-12s %16s  (%4.1f %%)  = %d x %s", "blocks", f"{sizes['block'] * sizes['blocks']:,d}",
             100 * sizes["block"] * sizes["blocks"] / sizes["total"], sizes["blocks"], f"{sizes['block']:,d}")
    log.info("Engine state per GPU in GB (resident / sharded schedule), before activations:")
    for gpus in (1, 2, 4, 8):
        plan = memory_plan(sizes, gpus)
        log.info("  %d GPU%s %8.1f / %8.1f", gpus, " " if gpus == 1 else "s", plan["resident"], plan["sharded"])
    return sizes


if __name__ == "__main__":
    prepare_cli_environment()
    if len(sys.argv) >= 2 and sys.argv[1] in ("-h", "--help"):
        print(f"{(__doc__ or '').strip()}\n\nUsage: {sys.argv[0]} CONFIG_PATH [--dotted.key=value ...]")
        sys.exit(0)
    if len(sys.argv) < 2:
        raise OLMoCliError(f"Usage: {sys.argv[0]} CONFIG_PATH [OPTIONS]")
    main(TrainConfig.load(sys.argv[1], [clean_opt(s) for s in sys.argv[2:]], validate_paths=False))
