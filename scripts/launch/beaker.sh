#!/usr/bin/env bash
# Entry point for a Beaker (or any batch scheduler that hands every replica the leader's host name and its own rank) job:
#   scripts/launch/beaker.sh CONFIG.yaml [--a.b=c ...]
# Beaker sets BEAKER_LEADER_REPLICA_HOSTNAME, BEAKER_REPLICA_RANK and BEAKER_REPLICA_COUNT inside a multi-replica
# experiment; with another scheduler export LEADER_HOST, NODE_RANK and NNODES instead.  Cloud credentials arrive as the
# secrets AWS_CONFIG / AWS_CREDENTIALS (file contents) and are written where the storage backends look for them.
# The job itself is scripts/launch/multi_node.sh: sharded inside a node, replicated across nodes, resuming from the newest
# checkpoint in the save folder so that a pre-empted experiment picks up where it stopped.
set -euo pipefail
CONFIG=$1; shift
export NNODES=${NNODES:-${BEAKER_REPLICA_COUNT:-1}}
export NODE_RANK=${NODE_RANK:-${BEAKER_REPLICA_RANK:-0}}
export MASTER_ADDR=${LEADER_HOST:-${BEAKER_LEADER_REPLICA_HOSTNAME:-127.0.0.1}}
if [[ -n "${AWS_CONFIG:-}" || -n "${AWS_CREDENTIALS:-}" ]]; then
  mkdir -p "$HOME/.aws"
  [[ -n "${AWS_CONFIG:-}" ]] && printenv AWS_CONFIG > "$HOME/.aws/config"
  [[ -n "${AWS_CREDENTIALS:-}" ]] && printenv AWS_CREDENTIALS > "$HOME/.aws/credentials"
fi
export OLMO_SHARED_FS=${OLMO_SHARED_FS:-1}        # replicas of one experiment mount the same checkpoint storage
here=$(dirname "$0")
if [[ "$NNODES" -le 1 ]]; then
  exec "$here/single_node.sh" "$CONFIG" "$@"
fi
exec "$here/multi_node.sh" "$CONFIG" "$@"
