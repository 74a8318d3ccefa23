#!/usr/bin/env bash
#SBATCH --job-name=dion-b200-1n
#SBATCH --nodes=1
#SBATCH --gpus-per-node=8
#SBATCH --ntasks-per-node=1
#SBATCH --exclusive
#SBATCH --time=12:00:00
#SBATCH --output=logs/%x_%j.out
# sbatch dion_b200/launch/slurm/job_single_node.sbatch <optimizer> [overrides...]
set -euo pipefail
source "$(dirname "$0")/env.sh" 2>/dev/null || source dion_b200/launch/slurm/env.sh
OPT=${1:-dion}
shift || true
NGPU=8 bash dion_b200/launch/run_single_node.sh "$OPT" "$@"
