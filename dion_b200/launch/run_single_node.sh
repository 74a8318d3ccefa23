#!/usr/bin/env bash
# Single-node FSDP training: one process per GPU, NCCL over NVLink.
#   NGPU=8 STEPS=10000 bash dion_b200/launch/run_single_node.sh <muon|dion|dion2|adamw|adadion|adadion_v2> [--section.field value ...]
# MODEL selects the config family (160m, 320m, 1b, 8b; default 160m).
set -euo pipefail
OPTIMIZER=${1:?"usage: $0 <muon|dion|dion2|adamw|adadion|adadion_v2> [overrides...]"}
shift
NGPU=${NGPU:-8}
STEPS=${STEPS:-10000}
MODEL=${MODEL:-160m}
MASTER_PORT=${MASTER_PORT:-29500}
CONFIG="llama3_${MODEL}_${OPTIMIZER}"
echo "=== single node: config=$CONFIG gpus=$NGPU steps=$STEPS ==="
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
export WANDB_RUN_NAME="${WANDB_RUN_NAME:-${OPTIMIZER}_${NGPU}gpu_${STEPS}steps}"
exec python -m torch.distributed.run --nnodes=1 --nproc-per-node="$NGPU" \
    --master-addr 127.0.0.1 --master-port "$MASTER_PORT" \
    -m dion_b200.train --config "$CONFIG" \
    --training.steps "$STEPS" \
    --parallelism.data_parallel_shard_degree "$NGPU" \
    --parallelism.data_parallel_replicate_degree 1 \
    "$@"
