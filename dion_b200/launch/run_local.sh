#!/usr/bin/env bash
# Validation without GPUs: NPROC CPU processes over gloo run the debug configs
# through the same trainer, optimizers and sharded code paths.
#   bash dion_b200/launch/run_local.sh [all|muon|dion|dion2|adamw|adadion|adadion_v2]
set -euo pipefail
WHICH=${1:-all}
STEPS=${STEPS:-3}
NPROC=${NPROC:-2}
MASTER_PORT=${MASTER_PORT:-29600}
run_test() {
    echo "--- $1 ---"
    CUDA_VISIBLE_DEVICES="" python -m torch.distributed.run --nnodes=1 --nproc-per-node="$NPROC" \
        --master-addr 127.0.0.1 --master-port "$MASTER_PORT" \
        -m dion_b200.train --config "$1" --training.steps "$STEPS" \
        --training.seq_len 64 --training.local_batch_size 2 --metrics.log_freq 1
    echo "--- $1: OK ---"
}
if [ "$WHICH" = "all" ]; then
    for o in muon dion dion2 adamw adadion adadion_v2; do run_test "llama3_debug_$o"; done
else
    run_test "llama3_debug_$WHICH"
fi
