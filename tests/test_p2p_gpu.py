"""In-kernel NVLink collectives (symmetric peer memory) against NCCL: the
fused Muon all-to-all and Dion reduce-scatter / all-gather paths must give
the same parameters as the NCCL paths. Needs 2+ GPUs on one node."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_collectives_match_nccl():
    n = min(torch.cuda.device_count(), 8)
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.path.dirname(here))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(here, "p2p_worker.py")]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert any(l.get("canaries_intact") for l in lines), "a kernel wrote outside a symmetric buffer"
    lines = [l for l in lines if "optimizer" in l]
    assert {l["optimizer"] for l in lines} == {"muon", "dion", "muon_ddp", "dion2"}
    for l in lines:
        assert l["status"] == 0
        assert l["max_abs_diff"] <= 1e-2 * l["max_abs"], l
