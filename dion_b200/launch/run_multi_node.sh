#!/usr/bin/env bash
# Multi-node HSDP training: shard within a node (NVLink), replicate across nodes.
# Run on every node with the same MASTER_ADDR / MASTER_PORT and its own NODE_RANK:
#   NUM_NODES=2 NODE_RANK=0 MASTER_ADDR=10.0.0.1 bash dion_b200/launch/run_multi_node.sh dion [overrides...]
set -euo pipefail
OPTIMIZER=${1:?"usage: $0 <muon|dion|dion2|adamw|adadion|adadion_v2> [overrides...]"}
shift
NUM_NODES=${NUM_NODES:-2}
NODE_RANK=${NODE_RANK:-0}
MASTER_ADDR=${MASTER_ADDR:?"MASTER_ADDR must be set for multi-node runs"}
MASTER_PORT=${MASTER_PORT:-29500}
GPUS_PER_NODE=${GPUS_PER_NODE:-8}
STEPS=${STEPS:-10000}
MODEL=${MODEL:-160m}
CONFIG="llama3_${MODEL}_${OPTIMIZER}"
echo "=== HSDP: config=$CONFIG nodes=$NUM_NODES x $GPUS_PER_NODE rank=$NODE_RANK master=$MASTER_ADDR:$MASTER_PORT ==="
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
export WANDB_RUN_NAME="${WANDB_RUN_NAME:-${OPTIMIZER}_$((NUM_NODES * GPUS_PER_NODE))gpu_hsdp_${STEPS}steps}"
exec python -m torch.distributed.run --nnodes="$NUM_NODES" --nproc-per-node="$GPUS_PER_NODE" \
    --node-rank="$NODE_RANK" --rdzv-backend=c10d --rdzv-endpoint="$MASTER_ADDR:$MASTER_PORT" \
    -m dion_b200.train --config "$CONFIG" \
    --training.steps "$STEPS" \
    --parallelism.data_parallel_shard_degree "$GPUS_PER_NODE" \
    --parallelism.data_parallel_replicate_degree "$NUM_NODES" \
    "$@"
