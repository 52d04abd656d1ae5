#!/usr/bin/env bash
# Train on every GPU of one B200 node:   scripts/launch/single_node.sh CONFIG.yaml [--a.b=c ...]
# One process per GPU; NVLink/NVSwitch collectives run through the framework's peer-memory kernels (FULL_SHARD) or NCCL.
set -euo pipefail
CONFIG=$1; shift
NGPU=${NGPU:-$(nvidia-smi -L | wc -l)}
export OMP_NUM_THREADS=${OMP_NUM_THREADS:-8}
export PYTHONFAULTHANDLER=1                 # stack traces of every thread on a fatal signal
export TORCH_DIST_INIT_BARRIER=1
export OLMO_SHARED_FS=${OLMO_SHARED_FS:-1}  # one node: every rank sees the same save folder
exec python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 --master-port "${MASTER_PORT:-29400}" \
  "$(dirname "$0")/../train.py" "$CONFIG" "$@"
