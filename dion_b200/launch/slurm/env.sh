#!/usr/bin/env bash
# Cluster environment shared by the sbatch files (source it; edit for your site).
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export OMP_NUM_THREADS=${OMP_NUM_THREADS:-8}
export DION_B200_P2P=${DION_B200_P2P:-1}
if [ -n "${SLURM_JOB_NODELIST:-}" ]; then
    MASTER_ADDR=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)
    export MASTER_ADDR
fi
export MASTER_PORT=${MASTER_PORT:-29500}
