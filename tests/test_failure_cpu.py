"""Failure handling made on the host (no device involved): non-finite and
all-zero gradients, checkpoint world-size mismatches, and ranks that stall
or leave between steps. (A rank that raises is covered in
test_distributed_cpu.py.)"""
import os
import time

import pytest
import torch
import torch.distributed as dist

from dion_b200.optim import AGDion, AdaDion, AdaDionV2, Dion, Dion2, GSDion, Muon, QCDion, SDion
from test_distributed_cpu import spawn

SMALL = dict(init_rank=4, rank_min=2, rank_max=16)
MAKERS = {
    "muon": lambda ps: Muon(ps, lr=0.02),
    "dion": lambda ps: Dion(ps, lr=0.02, rank_fraction=0.5),
    "dion2": lambda ps: Dion2(ps, lr=0.02, fraction=0.5),
    "adadion_v2": lambda ps: AdaDionV2(ps, lr=0.02, adaptive_rank=True, rank_min=2),
    "adadion": lambda ps: AdaDion(ps, lr=0.02, **SMALL),
    "sdion": lambda ps: SDion(ps, lr=0.02, **SMALL),
    "gsdion": lambda ps: GSDion(ps, lr=0.02, **SMALL),
    "agdion": lambda ps: AGDion(ps, lr=0.02, **SMALL),
    "qcdion": lambda ps: QCDion(ps, lr=0.02, **SMALL),
}
LOWRANK = ["dion", "adadion_v2", "adadion", "sdion", "gsdion", "agdion", "qcdion"]


def _params():
    torch.manual_seed(0)
    return [torch.nn.Parameter(torch.randn(24, 16)), torch.nn.Parameter(torch.randn(16, 40))]


@pytest.mark.parametrize("name", LOWRANK)
def test_zero_gradient_keeps_params_finite(name):
    """All-zero momentum makes the Gram / Cholesky factor singular: the guard must skip the update."""
    ps = _params()
    before = [p.detach().clone() for p in ps]
    opt = MAKERS[name](ps)
    for p in ps:
        p.grad = torch.zeros_like(p)
    opt.step()
    g = opt.param_groups[0]
    decay = 1.0 - float(g["lr"]) * float(g.get("weight_decay", 0.0))
    for p, b in zip(ps, before):
        assert torch.isfinite(p).all()
        # only (decoupled) weight decay may act on a zero gradient
        assert torch.allclose(p, b * decay, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["dion", "adadion_v2"])
def test_nan_gradient_is_discarded(name):
    ps = _params()
    opt = MAKERS[name](ps)
    for p in ps:
        p.grad = torch.randn_like(p)
    opt.step()
    ps[0].grad = torch.full_like(ps[0], float("nan"))
    ps[1].grad = torch.randn_like(ps[1])
    opt.step()
    assert all(torch.isfinite(p).all() for p in ps)


@pytest.mark.parametrize("name", ["adadion", "sdion", "gsdion", "agdion", "qcdion"])
def test_world_size_mismatch_on_load_raises(name):
    ps = _params()
    opt = MAKERS[name](ps)
    for p in ps:
        p.grad = torch.randn_like(p)
    opt.step()
    sd = opt.state_dict()
    # a checkpoint written by a 4-rank job (the stamp is only added when world_size > 1)
    sd[opt.WS_KEY] = 4
    with pytest.raises(RuntimeError, match="world_size"):
        MAKERS[name](_params()).load_state_dict(sd)


def _delayed(rank, world):
    if rank == 1:
        time.sleep(1.5)  # a slow rank: the others wait for it inside the collective
    t = torch.full((1,), float(rank + 1))
    dist.all_reduce(t)
    return float(t)


def test_delayed_rank_completes():
    out = spawn(_delayed)
    assert all(s == "ok" for s, _ in out.values()), out
    assert out[0][1] == out[1][1] == 3.0


def _leaver(rank, world):
    import datetime

    # a rank that leaves between steps: the others learn it through a short
    # process-group timeout on their next collective instead of hanging
    g = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=3))
    t = torch.ones(1)
    dist.all_reduce(t, group=g)  # step 1: everyone
    if rank == 1:
        return "left"
    t0 = time.time()
    try:
        dist.all_reduce(t, group=g)  # step 2: rank 1 is gone
    except Exception as e:  # noqa: BLE001
        raise RuntimeError(f"peer left after {time.time() - t0:.1f}s: {type(e).__name__}") from e
    return "no error"


def test_rank_leaving_between_steps_times_out():
    out = spawn(_leaver)
    assert out[1] == ("ok", "left")
    assert out[0][0] == "err" and "peer left" in out[0][1]


def test_elastic_restart_resumes_from_checkpoint(tmp_path):
    """A rank that raises mid-run (host-side) ends the attempt; torchrun's
    elastic agent restarts every rank and the job resumes from its last
    checkpoint and finishes (gloo, 2 ranks)."""
    import socket
    import subprocess
    import sys

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    here = os.path.dirname(os.path.abspath(__file__))
    ck = tmp_path / "ck"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--max-restarts=1",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(here, "elastic_worker.py"),
           "--config", "llama3_debug_muon", "--training.steps", "4", "--training.seq_len", "32",
           "--training.local_batch_size", "2", "--metrics.log_freq", "1", "--checkpoint.enable",
           "--checkpoint.folder", str(ck), "--checkpoint.interval", "2", "--checkpoint.no-last_save_model_only"]
    env = dict(os.environ, PYTHONPATH=os.path.dirname(here), CUDA_VISIBLE_DEVICES="")
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    log = res.stdout + res.stderr
    assert res.returncode == 0, log[-3000:]
    assert "injected host-side failure" in log
    steps = [int(l.split()[1]) for l in res.stdout.splitlines() if l.startswith("step:")]
    # attempt 1 logs steps 1-2 (then rank 1 fails); attempt 2 resumes at step 2 and logs 3-4
    assert steps == [1, 2, 3, 4], steps
    assert (ck / "step-2").exists() and (ck / "step-4").exists()
