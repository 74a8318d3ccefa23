#!/usr/bin/env bash
# Headline benchmark at 1, 2, 4 and 8 GPUs (both arms), one JSON line per run.
#   STEPS=10 WARMUP=3 bash dion_b200/launch/run_bench.sh [muon|dion]
set -euo pipefail
OPT=${1:-muon}
STEPS=${STEPS:-10}
WARMUP=${WARMUP:-3}
PORT=${MASTER_PORT:-29700}
for N in 1 2 4 8; do
    for IMPL in reference ours; do
        if [ "$N" = 1 ]; then
            python bench.py --gpus 1 --steps "$STEPS" --warmup "$WARMUP" --optimizer "$OPT" --impl "$IMPL"
        else
            timeout -k 60 1800 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$N" \
                --master-addr 127.0.0.1 --master-port "$PORT" \
                bench.py --gpus "$N" --steps "$STEPS" --warmup "$WARMUP" --optimizer "$OPT" --impl "$IMPL"
        fi
    done
done
