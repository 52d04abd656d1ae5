#!/usr/bin/env python
"""Write a default training config: ``scripts/init_config.py OUT.yaml [--dotted.key=value ...]``
(reference: ``scripts/init_config.py``)."""
import logging
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.config import TrainConfig
from olmo_b200.exceptions import OLMoCliError
from olmo_b200.util import clean_opt, prepare_cli_environment
from olmo_b200.utils import structured as S

log = logging.getLogger(__name__)


def main(save_path: Path, overrides) -> None:
    raw = S.deep_merge(S.to_container(TrainConfig()), S.parse_dotlist(overrides))
    cfg = S.build(TrainConfig, S.resolve_interpolations(raw))
    log.info("Saving config to %s", save_path)
    cfg.save(save_path)


if __name__ == "__main__":
    prepare_cli_environment()
    try:
        out, args = sys.argv[1], sys.argv[2:]
    except IndexError:
        raise OLMoCliError(f"Usage: {sys.argv[0]} [SAVE_PATH] [OPTIONS]")
    main(Path(out), [clean_opt(s) for s in args])
