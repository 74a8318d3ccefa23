#!/usr/bin/env bash
# The 33-run learning-rate x rank-fraction sweep on the 160M configs, one run
# after another on this node (logs/ and runs/ in the working directory).
#   STEPS=5000 NGPU=8 bash dion_b200/launch/run_sweep.sh
set -euo pipefail
STEPS=${STEPS:-5000}
NGPU=${NGPU:-8}
SCRIPT=$(mktemp)
python -m dion_b200.benchmarks.sweep --steps "$STEPS" --gpus "$NGPU" --script "$SCRIPT" > /dev/null
bash "$SCRIPT"
rm -f "$SCRIPT"
