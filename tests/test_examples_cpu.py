"""The examples in examples/ run on CPU: the plain training loop (loss falls
on a memorised batch) for each matrix optimizer, and the FSDP2 + Dion loop
as two gloo ranks under torch.distributed.run."""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("optimizer", ["muon", "dion", "dion2", "adadion_v2"])
def test_plain_pytorch_example(optimizer):
    sys.path.insert(0, os.path.join(ROOT, "examples"))
    try:
        import plain_pytorch
    finally:
        sys.path.pop(0)
    losses = plain_pytorch.main(["--optimizer", optimizer, "--steps", "12", "--device", "cpu"])
    assert losses[-1] < losses[0] - 0.5, losses


def test_fsdp_example_two_ranks():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(port), os.path.join(ROOT, "examples", "fsdp_dion.py"), "--steps", "3"]
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert res.returncode == 0, (res.stdout + res.stderr)[-3000:]
    steps = [l for l in res.stdout.splitlines() if l.startswith("step")]
    assert len(steps) == 2 and float(steps[-1].split()[-1]) < float(steps[0].split()[-1])
