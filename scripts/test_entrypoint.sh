#!/usr/bin/env bash
# Entry point of a test or benchmark job in a container:  scripts/test_entrypoint.sh CMD [ARGS...]
# Builds the kernel library for sm_100a if it is missing or stale, then runs the command with its output copied to
# $RESULTS_DIR/out.log (default /results).  The exit status is the command's.
set -euo pipefail
if [[ $# -eq 0 ]]; then
  echo >&2 "usage: $0 CMD [ARGS...]"; exit 2
fi
REPO=$(cd "$(dirname "$0")/.." && pwd)
RESULTS_DIR=${RESULTS_DIR:-/results}
mkdir -p "$RESULTS_DIR"
cd "$REPO"
python -m olmo_b200.ops 2>&1 | tee "$RESULTS_DIR/build.log"
"$@" 2>&1 | tee "$RESULTS_DIR/out.log"
