#!/usr/bin/env bash
# One launcher for the published OLMo-2 ("peteish") runs and their follow-ups, on any cluster:
#
#   scripts/launch/published_runs.sh RUN [--a.b=c ...]
#
#   RUN                     what it trains
#   peteish1|7|13           the 1B / 7B / 13B pre-training runs
#   peteish7-medlr          7B at the lower peak learning rate (6e-4)
#   peteish13-medlr|-highlr 13B at 6e-4 / 9e-4
#   peteish7-lr-anneal      7B: linear decay to zero from a step of an earlier run (START_STEP, ANNEAL_TOKENS, START_LR, LOAD_PATH)
#   anneal                  a data anneal from its own config (CONFIG=configs/annealing/....yaml [SEED=...])
#   tiny                    a model of the small family (SIZE=20M|60M|150M|300M|700M)
#   ladder                  a scaling-ladder run: everything after RUN goes to scripts/ladder.py train
#   unshard                 sharded checkpoint -> unsharded: scripts/unshard.py with the remaining arguments
#
# Environment: STORAGE=google|weka|s3 (which copy of the token files the config points at; default weka),
# CHECKPOINT_ROOT (local or mounted folder for checkpoints; default ./runs), REMOTE_ROOT (optional URL prefix mirrored to),
# NAME (run name; default RUN), plus what scripts/launch/beaker.sh reads for the node layout (NNODES, NODE_RANK,
# LEADER_HOST or the Beaker variables).  Across nodes the model is sharded inside a node and replicated between nodes,
# and a restarted job resumes from the newest checkpoint under its save folder.
# The reference keeps one pair of shell scripts per run and cluster (scripts/beaker/peteish/*.sh, scripts/augusta/*.sh);
# the settings those scripts pass on the command line are the table below.
set -euo pipefail
RUN=${1:?usage: published_runs.sh RUN [overrides]}; shift
here=$(cd "$(dirname "$0")" && pwd)
repo=$(cd "$here/../.." && pwd)
STORAGE=${STORAGE:-weka}
NAME=${NAME:-$RUN}
CHECKPOINT_ROOT=${CHECKPOINT_ROOT:-$repo/runs}
NNODES=${NNODES:-${BEAKER_REPLICA_COUNT:-1}}

case "$RUN" in
  ladder)  exec python "$repo/scripts/ladder.py" train "$@" ;;
  unshard) exec python "$repo/scripts/unshard.py" "$@" ;;
esac

config=""           # YAML below configs/
settings=()         # dotted overrides of that run
case "$RUN" in
  peteish1)
    config=peteish1-$STORAGE.yaml
    settings=(--device_train_microbatch_size=4 --save_interval_ephemeral=10000 --eval_interval=10000 --data.num_workers=32) ;;
  peteish7)
    config=peteish7-$STORAGE.yaml
    settings=(--device_train_microbatch_size=2 --save_interval_ephemeral=1000 --eval_interval=1000) ;;
  peteish7-medlr)
    config=peteish7-$STORAGE.yaml
    settings=(--device_train_microbatch_size=2 --activation_checkpointing=one_in_four --optimizer.learning_rate=6.0e-4
              --save_interval_ephemeral=1000 --eval_interval=1000) ;;
  peteish7-lr-anneal)
    # From step START_STEP of an earlier run, decay the learning rate linearly to zero over ANNEAL_TOKENS tokens.  START_LR and
    # LOAD_PATH are given, or looked up from the earlier run's W&B record (ORIGINAL_WANDB_RUN_ID) under REMOTE_ROOT.
    : "${START_STEP:?set START_STEP (and START_LR + LOAD_PATH, or ORIGINAL_WANDB_RUN_ID + REMOTE_ROOT)}"
    if [[ -n "${ORIGINAL_WANDB_RUN_ID:-}" ]]; then
      START_LR=${START_LR:-$(python "$repo/scripts/learning_rate_at_step_from_wandb.py" "$ORIGINAL_WANDB_RUN_ID" "$START_STEP")}
      LOAD_PATH=${LOAD_PATH:-${REMOTE_ROOT:?}/$(python "$repo/scripts/group_name_from_wandb.py" "$ORIGINAL_WANDB_RUN_ID")/step$START_STEP}
    fi
    : "${START_LR:?}" "${LOAD_PATH:?}"
    last_step=$(python -c "print(round(${ANNEAL_TOKENS:-50e9} / (1024 * 4096)) + $START_STEP)")
    config=peteish7-$STORAGE.yaml
    settings=(--device_train_microbatch_size=2 --activation_checkpointing=one_in_four "--load_path=$LOAD_PATH"
              "--optimizer.learning_rate=$START_LR" --scheduler.units=steps --scheduler.name=linear_with_warmup
              "--scheduler.t_warmup=$START_STEP" --scheduler.t_max=null --scheduler.alpha_f=0
              "--max_duration=$last_step" "--stop_at=$((last_step + 10))" --no_pre_train_checkpoint
              --save_interval_ephemeral=1000 --eval_interval=1000) ;;
  peteish13)
    config=peteish13-$STORAGE.yaml
    settings=(--device_train_microbatch_size=2 --activation_checkpointing=one_in_two --optimizer.learning_rate=9.0e-4
              --save_interval_ephemeral=1000 --save_num_checkpoints_to_keep=2 --eval_interval=1000) ;;
  peteish13-medlr)
    config=peteish13-$STORAGE.yaml
    settings=(--device_train_microbatch_size=2 --activation_checkpointing=one_in_two --optimizer.learning_rate=6.0e-4
              --save_interval_ephemeral=1000 --eval_interval=1000) ;;
  peteish13-highlr)
    config=peteish13-$STORAGE.yaml
    settings=(--device_train_microbatch_size=2 --activation_checkpointing=one_in_two --optimizer.learning_rate=9.0e-4
              --save_interval_ephemeral=1000 --eval_interval=1000) ;;
  anneal)
    config=${CONFIG:?set CONFIG to the anneal YAML}
    settings=(--device_train_microbatch_size=2 --activation_checkpointing=one_in_four --no_pre_train_checkpoint
              --save_interval_ephemeral=1000 --eval_interval=1000)
    [[ -n "${SEED:-}" ]] && settings+=("--seed=$SEED") ;;
  tiny)
    config=tiny/OLMo-${SIZE:-20M}.yaml
    settings=(--save_interval_ephemeral=null) ;;
  *)
    echo "unknown run '$RUN' (see the table at the top of $0)" >&2; exit 2 ;;
esac
[[ "$config" = /* || -f "$config" ]] || config="$repo/configs/$config"
[[ -f "$config" ]] || { echo "no such config: $config" >&2; exit 2; }

common=("--run_name=$NAME" "--save_folder=$CHECKPOINT_ROOT/$NAME" --save_overwrite --optimizer.metrics_log_interval=10
        --data.prefetch_factor=8)
[[ -n "${REMOTE_ROOT:-}" ]] && common+=("--remote_save_folder=${REMOTE_ROOT%/}/$NAME/")
[[ -n "${WANDB_API_KEY:-}" ]] && common+=("--wandb.group=$NAME")
# a restarted job continues from the newest checkpoint under its save folder (or its mirror); only when there is none
# does a --load_path from the table or from the caller apply
common+=(--try_load_latest_save)
if [[ "$NNODES" -gt 1 ]]; then
  common+=(--fsdp.sharding_strategy=HYBRID_SHARD "--fsdp.hybrid_sharding_num_model_replicas=$NNODES")
fi

if [[ -n "${DRY_RUN:-}" ]]; then
  printf '%s\n' "$here/beaker.sh" "$config" "${settings[@]}" "${common[@]}" "$@"
  exit 0
fi
exec "$here/beaker.sh" "$config" "${settings[@]}" "${common[@]}" "$@"
