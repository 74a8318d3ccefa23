"""Sequence-parallel TP collectives on CPU (gloo, 2 ranks): ``SPGroup``'s
all-gather and GEMM -> reduce-scatter, and the autograd functions built on
them, must equal the same products computed on the full, unsharded tensors.
The multi-GPU peer-memory form of the same functions is checked in
tests/test_parallel_gpu.py and tests/test_sp_emulated_gpu.py."""
import functools

import pytest
import torch

from test_distributed_cpu import spawn


def _collectives_body(rank, world):
    import torch.distributed as dist

    from dion_b200.parallel.sp import SPGroup

    sp = SPGroup(dist.group.WORLD, torch.device("cpu"))
    assert not sp.p2p and sp.T == world and sp.me == rank
    g = torch.Generator().manual_seed(0)
    N, K, D = 8 * world, 6, 5
    full = torch.randn(N, D, generator=g)
    gathered = sp.all_gather(sp.shard_rows(full))
    # every rank's partial product; the reduce-scatter returns row block `rank` of their sum
    A = [torch.randn(N, K, generator=g) for _ in range(world)]
    B = [torch.randn(K, D, generator=g) for _ in range(world)]
    rs = sp.gemm_reduce_scatter(A[rank], B[rank])
    ref = sum(a @ b for a, b in zip(A, B))
    n = N // world
    return [float((gathered - full).abs().max()), float((rs - ref[rank * n:(rank + 1) * n]).abs().max())]


def test_sp_all_gather_and_gemm_reduce_scatter():
    out = spawn(_collectives_body, world=2)
    for r, (status, res) in out.items():
        assert status == "ok", res
        assert res[0] == 0.0
        assert res[1] < 1e-5


def _autograd_body(rank, world):
    """A column-parallel pair then a row-parallel linear, on a token shard,
    against the unsharded two-layer product and its gradients."""
    import torch.distributed as dist

    from dion_b200.parallel.sp import SPGroup, sp_column_linears, sp_row_linear

    sp = SPGroup(dist.group.WORLD, torch.device("cpu"))
    g = torch.Generator().manual_seed(1)
    N, D, H = 4 * world, 8, 6 * world
    x = torch.randn(N, D, generator=g)
    W1 = torch.randn(H, D, generator=g)
    W3 = torch.randn(H, D, generator=g)
    W2 = torch.randn(D, H, generator=g)
    dy = torch.randn(N, D, generator=g)

    # reference on the full tensors
    xr, W1r, W3r, W2r = (t.clone().requires_grad_() for t in (x, W1, W3, W2))
    yr = ((xr @ W1r.t()) * (xr @ W3r.t())) @ W2r.t()
    yr.backward(dy)

    # TP: rank r holds rows [r*h, (r+1)*h) of W1/W3 and the matching columns of W2
    h = H // world
    cols = slice(rank * h, (rank + 1) * h)
    xs = sp.shard_rows(x).clone().requires_grad_()
    w1 = W1[cols].clone().requires_grad_()
    w3 = W3[cols].clone().requires_grad_()
    w2 = W2[:, cols].clone().requires_grad_()
    a, b = sp_column_linears(sp, xs, [w1, w3])
    ys = sp_row_linear(sp, a * b, w2)
    ys.backward(sp.shard_rows(dy))

    def err(u, v):
        return float((u - v).abs().max() / v.abs().max())

    return [err(ys.detach(), sp.shard_rows(yr.detach())), err(xs.grad, sp.shard_rows(xr.grad)),
            err(w1.grad, W1r.grad[cols]), err(w3.grad, W3r.grad[cols]), err(w2.grad, W2r.grad[:, cols])]


def test_sp_linears_forward_backward():
    out = spawn(_autograd_body, world=2)
    for r, (status, res) in out.items():
        assert status == "ok", res
        assert max(res) < 1e-5, res


def _train_body(sequence_parallel, dp_shard, tp, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name="Muon", lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64),
                        seq_len=32, local_batch_size=2, steps=3, warmup_steps=0, dp_shard=dp_shard, tp=tp,
                        optimizer=opt, seed=5, sequence_parallel=sequence_parallel)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    assert (getattr(tr.model, "sp", None) is not None) == (sequence_parallel and tp > 1)
    losses = []
    for _ in range(3):
        t, l = tr.data.next()
        losses.append(float(tr.train_step(t, l)))
    return losses


@pytest.mark.parametrize("sequence_parallel", [False, True])
def test_tp_matches_single_process(sequence_parallel):
    """TP 2 (with and without sequence parallelism) against one process on
    the same batch: TP ranks see the same sequences, so the losses agree."""
    ref = spawn(functools.partial(_train_body, False, 1, 1), world=1)
    got = spawn(functools.partial(_train_body, sequence_parallel, 1, 2), world=2)
    for out in (ref, got):
        for r, (status, res) in out.items():
            assert status == "ok", res
    a = torch.tensor(ref[0][1])
    b = torch.tensor(got[0][1])
    assert torch.isfinite(b).all()
    assert torch.allclose(a, b, rtol=2e-3, atol=2e-3), (a, b)


def _accum_body(local, global_batch, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=local, global_batch_size=global_batch, steps=3, warmup_steps=0, dp_shard=1,
                        tp=2, optimizer=HybridOptimizersContainer.Config(name="Muon", lr=0.02), seed=5)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    return [float(tr.train_step(*tr.data.next())) for _ in range(3)]


def test_gradient_accumulation_with_sequence_parallel_tp():
    """TP 2 (sequence parallel): two accumulated micro-batches of 2 train like
    one batch of 4 (the TP sum of replicated gradients runs once per step)."""
    full = spawn(functools.partial(_accum_body, 4, 4), world=2)
    acc = spawn(functools.partial(_accum_body, 2, 4), world=2)
    for out in (full, acc):
        for r, (status, res) in out.items():
            assert status == "ok", res
    a, b = torch.tensor(full[0][1]), torch.tensor(acc[0][1])
    assert torch.allclose(a, b, rtol=1e-4, atol=1e-4), (a, b)


def _odd_tokens_body(rank, world):
    import torch.distributed as dist

    from dion_b200.parallel.sp import SPGroup

    sp = SPGroup(dist.group.WORLD, torch.device("cpu"))
    try:
        sp.shard_rows(torch.zeros(7, 4))
    except ValueError as e:
        return [str(e)]
    return ["no error"]


def test_token_count_must_divide_over_tp_ranks():
    out = spawn(_odd_tokens_body, world=2)
    for r, (status, res) in out.items():
        assert status == "ok", res
        assert "multiple of 2" in res[0], res
