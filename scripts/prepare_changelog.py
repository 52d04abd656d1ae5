#!/usr/bin/env python
"""Move the "Unreleased" entries of ``CHANGELOG.md`` under the version in ``olmo_b200/version.py`` (the reference's script of
this name; here a shorthand for ``python scripts/release.py stamp``)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from release import main

if __name__ == "__main__":
    sys.exit(main(["stamp", *sys.argv[1:]]))  # no options of its own: anything else (``--help`` too) goes to the parser
