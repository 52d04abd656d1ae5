#!/usr/bin/env bash
# Train on several B200 nodes (run once per node):
#   NNODES=4 NODE_RANK=0 MASTER_ADDR=10.0.0.1 scripts/launch/multi_node.sh CONFIG.yaml [--a.b=c ...]
# Parameters are sharded inside a node (NVSwitch) and replicated across nodes (HYBRID_SHARD): the cross-node link only
# carries the all-reduce of already reduce-scattered gradient shards.
set -euo pipefail
CONFIG=$1; shift
: "${NNODES:?set NNODES}" "${NODE_RANK:?set NODE_RANK}" "${MASTER_ADDR:?set MASTER_ADDR}"
NGPU=${NGPU:-$(nvidia-smi -L | wc -l)}
export OMP_NUM_THREADS=${OMP_NUM_THREADS:-8}
export PYTHONFAULTHANDLER=1
export TORCH_DIST_INIT_BARRIER=1
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export NCCL_IB_TIMEOUT=${NCCL_IB_TIMEOUT:-22}     # ride out short fabric hiccups instead of aborting the job
export TORCH_NCCL_ASYNC_ERROR_HANDLING=1          # a failed collective raises on the host instead of hanging the rank
exec python -m torch.distributed.run --nnodes "$NNODES" --node-rank "$NODE_RANK" --nproc-per-node "$NGPU" \
  --rdzv-backend static --master-addr "$MASTER_ADDR" --master-port "${MASTER_PORT:-29400}" \
  "$(dirname "$0")/../train.py" "$CONFIG" \
  --fsdp.sharding_strategy=HYBRID_SHARD --fsdp.hybrid_sharding_num_model_replicas="$NNODES" \
  --load_path='${path.last_checkpoint:${save_folder}}' --try_load_latest_save=true "$@"
