#!/usr/bin/env bash
# Multi-node training under Slurm, one task per node, one process per GPU inside it:
#   sbatch --nodes=4 scripts/launch/slurm.sbatch configs/official-1124/OLMo2-13B-stage1.yaml --save_folder=/shared/runs/13b
# HYBRID_SHARD keeps parameter all-gathers and gradient reduce-scatters inside a node (NVLink peer memory) and only
# all-reduces the sharded gradients between nodes; the number of model replicas defaults to the number of nodes.
#SBATCH --job-name=olmo-b200
#SBATCH --ntasks-per-node=1
#SBATCH --gpus-per-node=8
#SBATCH --cpus-per-task=64
#SBATCH --exclusive
set -euo pipefail
CONFIG=$1; shift
REPO=$(cd "$(dirname "$0")/../.." && pwd)
export MASTER_ADDR=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)
export MASTER_PORT=${MASTER_PORT:-29400}
export OMP_NUM_THREADS=${OMP_NUM_THREADS:-8}
export PYTHONFAULTHANDLER=1
export OLMO_SHARED_FS=${OLMO_SHARED_FS:-1}   # save_folder is on a file system every node sees
NGPU=${NGPU:-8}
srun --kill-on-bad-exit=1 bash -c "
  python -m torch.distributed.run --nnodes=\$SLURM_NNODES --node-rank=\$SLURM_NODEID --nproc-per-node=$NGPU \
    --rdzv-backend=static --master-addr=\$MASTER_ADDR --master-port=\$MASTER_PORT \
    $REPO/scripts/train.py $CONFIG \
    --fsdp.sharding_strategy=HYBRID_SHARD --fsdp.hybrid_sharding_num_model_replicas=\$SLURM_NNODES $*"
