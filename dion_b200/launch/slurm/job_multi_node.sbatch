#!/usr/bin/env bash
#SBATCH --job-name=dion-b200-hsdp
#SBATCH --nodes=2
#SBATCH --gpus-per-node=8
#SBATCH --ntasks-per-node=1
#SBATCH --exclusive
#SBATCH --time=12:00:00
#SBATCH --output=logs/%x_%j.out
# sbatch --nodes=N dion_b200/launch/slurm/job_multi_node.sbatch <optimizer> [overrides...]
set -euo pipefail
source "$(dirname "$0")/env.sh" 2>/dev/null || source dion_b200/launch/slurm/env.sh
OPT=${1:-dion}
shift || true
srun --kill-on-bad-exit=1 bash -c "NUM_NODES=$SLURM_JOB_NUM_NODES NODE_RANK=\$SLURM_NODEID \
    bash dion_b200/launch/run_multi_node.sh $OPT $*"
