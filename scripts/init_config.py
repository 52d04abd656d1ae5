#!/usr/bin/env python
"""Write a starting training config.

    scripts/init_config.py OUT.yaml [--from RECIPE] [--dotted.key=value ...]
    scripts/init_config.py --list

Without ``--from`` the file holds the defaults of every field (what the reference's ``scripts/init_config.py`` writes);
with it, the named recipe of ``olmo_b200.recipes`` (an official OLMo / OLMo-2 run, a tiny model, ...).  Dotted overrides are
applied on top and the result is validated before it is written.
"""
import logging
import sys
from pathlib import Path
from typing import List, Optional

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from olmo_b200.config import TrainConfig
from olmo_b200.exceptions import OLMoCliError
from olmo_b200.util import clean_opt, prepare_cli_environment
from olmo_b200.utils import structured as S

log = logging.getLogger(__name__)


def main(save_path: Path, overrides: List[str], recipe: Optional[str] = None) -> TrainConfig:
    if recipe is None:
        merged = S.deep_merge(S.to_container(TrainConfig()), S.parse_dotlist(overrides))
        cfg = S.build(TrainConfig, S.resolve_interpolations(merged))
    else:
        from olmo_b200.recipes import RECIPES, recipe_config

        if recipe not in RECIPES:
            raise OLMoCliError(f"unknown recipe '{recipe}'; `--list` shows the names")
        cfg = recipe_config(recipe, overrides)
    cfg.save(save_path)
    log.info("wrote %s (%s)", save_path, f"recipe {recipe}" if recipe else "field defaults")
    return cfg


if __name__ == "__main__":
    prepare_cli_environment()
    argv = sys.argv[1:]
    if "-h" in argv or "--help" in argv:
        print((__doc__ or "").strip())
        sys.exit(0)
    if "--list" in argv:
        from olmo_b200.recipes import RECIPES

        print("\n".join(sorted(RECIPES)))
        sys.exit(0)
    recipe = None
    if "--from" in argv:
        at = argv.index("--from")
        if at + 1 >= len(argv):
            raise OLMoCliError("--from needs a recipe name")
        recipe = argv[at + 1]
        del argv[at : at + 2]
    if not argv:
        raise OLMoCliError(f"Usage: {sys.argv[0]} SAVE_PATH [--from RECIPE] [OPTIONS]")
    if argv[0].startswith("-"):
        raise OLMoCliError(f"the first argument is the file to write, not an option ('{argv[0]}')")
    main(Path(argv[0]), [clean_opt(s) for s in argv[1:]], recipe)
