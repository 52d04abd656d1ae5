#!/usr/bin/env python
"""Print the parameter counts of the model described by a training config:
``scripts/show_model_size.py CONFIG.yaml [--model.key=value ...]`` (reference: ``scripts/show_model_size.py``)."""
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.config import TrainConfig
from olmo_b200.exceptions import OLMoCliError
from olmo_b200.models.olmo import OLMo
from olmo_b200.util import clean_opt, prepare_cli_environment

log = logging.getLogger(__name__)


def main(cfg: TrainConfig) -> None:
    cfg.model.init_device = "meta"  # counting needs no storage
    n_layers = cfg.model.n_layers
    cfg.model.n_layers = 1
    single = OLMo(cfg.model, init_params=False)
    block = sum(p.numel() for p in single.transformer.blocks.parameters())  # type: ignore[union-attr]
    total = single.num_params() + block * (n_layers - 1)
    non_emb = single.num_params(include_embedding=False) + block * (n_layers - 1)
    log.info("Total number of parameters: %s", f"{total:,d}")
    log.info("Number of non-embedding parameters: %s", f"{non_emb:,d}")


if __name__ == "__main__":
    prepare_cli_environment()
    try:
        yaml_path, overrides = sys.argv[1], sys.argv[2:]
    except IndexError:
        raise OLMoCliError(f"Usage: {sys.argv[0]} [CONFIG_PATH] [OPTIONS]")
    main(TrainConfig.load(yaml_path, [clean_opt(s) for s in overrides], validate_paths=False))
