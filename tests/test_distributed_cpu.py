"""Multi-process (gloo, world size 2) checks of the sharded optimizer paths:
FSDP-sharded Muon / Dion / Dion2 / AdaDionV2 must produce the same
parameters as the single-process run on the full matrices, DDP Muon must
agree across replicas, and a rank that raises must surface as an error on
the others (host-side failure, no device involved)."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import datetime

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        res = fn(rank, world)
        if isinstance(res, list):
            res = [t.tolist() if isinstance(t, torch.Tensor) else t for t in res]
        q.put((rank, "ok", res))
    except Exception:
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def spawn(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, res = q.get(timeout=120)
        if status == "ok" and isinstance(res, list):
            res = [torch.tensor(t) if isinstance(t, list) else t for t in res]
        out[r] = (status, res)
    for p in procs:
        p.join(timeout=60)
    return out


SHAPES = [(8, 12), (8, 12), (8, 12), (16, 8), (16, 8)]
# Dion orients by the sharding under FSDP (row-sharded => transposed), so the
# single-process comparison uses wide matrices, where both layouts agree
WIDE = [(8, 12), (8, 12), (8, 12), (8, 16), (8, 16)]


def _params(seed=0, shapes=None):
    g = torch.Generator().manual_seed(seed)
    shapes = shapes or SHAPES
    X = [torch.randn(s, generator=g) for s in shapes]
    G = [torch.randn(s, generator=g) for s in shapes]
    return X, G


def _make(name, params, mesh):
    from dion_b200.optim import AdaDionV2, Dion, Dion2, Muon

    if name == "muon":
        return Muon(params, distributed_mesh=mesh, lr=0.05, mu=0.9, weight_decay=0.1, ns_coeffs="keller")
    if name == "dion":
        return Dion(params, outer_shard_mesh=mesh, lr=0.05, mu=0.9, weight_decay=0.1, rank_fraction=0.5)
    if name == "dion2":
        return Dion2(params, distributed_mesh=mesh, lr=0.05, fraction=0.5, weight_decay=0.1)
    return AdaDionV2(params, outer_shard_mesh=mesh, lr=0.05, mu=0.9, rank_fraction_max=0.5)


def _sharded_fn(name, rank, world):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    mesh = init_device_mesh("cpu", (world,))
    X, G = _params(shapes=WIDE if name in ("dion", "adadion_v2") else None)
    torch.manual_seed(123)  # identical Q draws on every rank
    ps = [torch.nn.Parameter(distribute_tensor(x.clone(), mesh, [Shard(0)])) for x in X]
    for p, g in zip(ps, G):
        p.grad = distribute_tensor(g.clone(), mesh, [Shard(0)])
    opt = _make(name, ps, mesh)
    for _ in range(2):
        opt.step()
    return [p.full_tensor().detach() for p in ps]


def _sharded_step(name):
    import functools

    return functools.partial(_sharded_fn, name)


def _single(name):
    X, G = _params(shapes=WIDE if name in ("dion", "adadion_v2") else None)
    torch.manual_seed(123)
    ps = [torch.nn.Parameter(x.clone()) for x in X]
    for p, g in zip(ps, G):
        p.grad = g.clone()
    opt = _make(name, ps, None)
    for _ in range(2):
        opt.step()
    return [p.detach() for p in ps]


@pytest.mark.parametrize("name", ["muon", "dion", "dion2", "adadion_v2"])
def test_fsdp_matches_single_process(name):
    out = spawn(_sharded_step(name))
    for r, (status, res) in out.items():
        assert status == "ok", res
    ref = _single(name)
    for a, b in zip(out[0][1], out[1][1]):
        torch.testing.assert_close(a, b)
    if name == "dion2":
        # per-shard row selection differs from a global top-k by design: check the step ran and moved params
        X, _ = _params()
        assert all(not torch.equal(a, x) for a, x in zip(out[0][1], X))
        return
    if name in ("dion", "adadion_v2"):
        # sketch draws differ between layouts; the update is invariant up to the orthogonalisation
        for a, b in zip(out[0][1], ref):
            torch.testing.assert_close(a, b, rtol=2e-3, atol=2e-3)
        return
    for a, b in zip(out[0][1], ref):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-3)


def _ddp_muon(rank, world):
    from dion_b200.optim import Muon

    X, G = _params()
    ps = [torch.nn.Parameter(x.clone()) for x in X]
    for p, g in zip(ps, G):
        p.grad = g.clone()
    opt = Muon(ps, distributed_mesh=dist.group.WORLD, lr=0.05, ns_coeffs="keller")
    opt.step()
    return [p.detach() for p in ps]


def test_ddp_muon_replicas_agree():
    out = spawn(_ddp_muon)
    assert all(s == "ok" for s, _ in out.values()), out
    for a, b in zip(out[0][1], out[1][1]):
        torch.testing.assert_close(a, b)


def _failing(rank, world):
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    t = torch.ones(1)
    dist.all_reduce(t)  # rank 1 never joins: gloo times out / sees the peer leave
    return float(t)


def test_rank_failure_surfaces_on_host():
    out = spawn(_failing)
    assert out[1][0] == "err" and "injected failure" in out[1][1]
    assert out[0][0] == "err"
