#!/usr/bin/env bash
# Prepare a node to run dion_b200: build the in-tree extensions (sm_100a kernels and the
# host-side data loader), check that they import, and report the GPUs, NCCL and the
# environment the launchers use. Run it once per node (no network access is needed).
#
#   bash dion_b200/launch/setup_env.sh            # build + checks
#   SKIP_BUILD=1 bash dion_b200/launch/setup_env.sh
set -euo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)"
cd "$ROOT"
PY=${PYTHON:-python}

if [ -z "${SKIP_BUILD:-}" ]; then
    echo "=== building extensions (nvcc -gencode arch=compute_100a,code=sm_100a) ==="
    MAX_JOBS=${MAX_JOBS:-$(nproc)} "$PY" setup.py build_ext --inplace > build_ext.log 2>&1 \
        || { echo "build failed: see $ROOT/build_ext.log"; exit 1; }
fi

echo "=== imports ==="
"$PY" - <<'EOF'
import torch
import dion_b200, dion_b200._C, dion_b200._io  # noqa: F401  (both native libraries must load)
from dion_b200 import ops
print(f"torch {torch.__version__}  cuda {torch.version.cuda}  nccl {'.'.join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else '-'}")
print(f"extension loaded: {ops.has_ext()}")
n = torch.cuda.device_count()
print(f"GPUs: {n}")
for i in range(n):
    p = torch.cuda.get_device_properties(i)
    print(f"  cuda:{i} {p.name} sm_{p.major}{p.minor} {p.total_memory / 2**30:.0f} GiB {p.multi_processor_count} SMs")
    if (p.major, p.minor) != (10, 0):
        print("  warning: the kernels are built for sm_100a (B200); this GPU cannot run them")
if n > 1:
    peer = all(torch.cuda.can_device_access_peer(i, j) for i in range(n) for j in range(n) if i != j)
    print(f"peer access between all GPUs: {peer} (the fused collectives need it; else they use NCCL)")
EOF

echo "=== environment ==="
echo "PYTORCH_CUDA_ALLOC_CONF=${PYTORCH_CUDA_ALLOC_CONF:-<unset; launchers set expandable_segments:True>}"
echo "DION_B200_P2P=${DION_B200_P2P:-<unset: peer-memory collectives on one node>}"
echo "NCCL_DEBUG=${NCCL_DEBUG:-<unset>}"
echo "ok"
