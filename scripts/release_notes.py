#!/usr/bin/env python
"""Print the release notes of one version: ``python scripts/release_notes.py v0.6.0`` (the reference's script of this name;
here a shorthand for ``python scripts/release.py notes VERSION``)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from release import main

if __name__ == "__main__":
    sys.exit(main(["notes", *sys.argv[1:]]))
