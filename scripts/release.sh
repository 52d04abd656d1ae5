#!/usr/bin/env bash
# Tag a release: stamps CHANGELOG.md with the version in olmo_b200/version.py, commits it, creates and pushes the tag
# (asks before doing anything).  Shorthand for `python scripts/release.py tag`.
set -euo pipefail
exec python "$(dirname "$0")/release.py" tag "$@"
