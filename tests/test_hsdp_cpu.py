"""HSDP on CPU (gloo, 4 ranks = 2 replicas x 2 shards): Muon and Dion2 give
the losses of plain FSDP over 4 ranks on the same global batch; Dion (whose
replicas synchronise the low-rank factors instead of gradients when that is
cheaper) and AdamW train."""
import functools

import pytest
import torch

from test_distributed_cpu import spawn


def _body(optimizer, replicate, shard, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=2, steps=3, warmup_steps=0, dp_replicate=replicate, dp_shard=shard,
                        optimizer=opt, seed=11)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    out = []
    for _ in range(3):
        t, l = tr.data.next()
        out.append(float(tr.train_step(t, l)))
    return out


def _run(optimizer, replicate, shard):
    res = spawn(functools.partial(_body, optimizer, replicate, shard), world=replicate * shard)
    for r in res.values():
        assert r[0] == "ok", r[1]
    return torch.tensor(res[0][1])


@pytest.mark.parametrize("optimizer", ["Muon", "Dion2"])
def test_hsdp_matches_fsdp(optimizer):
    ref = _run(optimizer, 1, 4)
    got = _run(optimizer, 2, 2)
    assert torch.allclose(ref, got, rtol=2e-3, atol=2e-3), (ref, got)


@pytest.mark.parametrize("optimizer", ["Dion", "AdamW"])
def test_hsdp_trains(optimizer):
    got = _run(optimizer, 2, 2)
    assert torch.isfinite(got).all()


def _ckpt_body(folder, phase, optimizer, rank, world):
    import torch.distributed as dist

    from dion_b200.checkpoint import CheckpointManager
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=2, steps=4, warmup_steps=0, dp_replicate=2, dp_shard=2, optimizer=opt,
                        seed=11)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    ck = CheckpointManager(folder, tr.model, tr.optimizers, interval=2, model_only_last=False)
    if phase == "save":
        for s in (1, 2):
            tr.train_step(*tr.data.next())
            ck.maybe_save(tr, s)
    else:
        ck.maybe_load(tr)
        assert tr.step_idx == 2
    out = []
    for _ in range(2):
        loss = tr.train_step(*tr.data.next()).detach().clone()
        dist.all_reduce(loss)
        out.append(float(loss / world))
    return out


@pytest.mark.parametrize("optimizer", ["Dion", "Muon", "AdaDionV2", "AdaDion"])
def test_hsdp_checkpoint_resume(tmp_path, optimizer):
    """HSDP 2 x 2: replicas synchronise their state before the save
    (Dion's ``synchronize_for_checkpoint``), and the resumed run continues
    with the uninterrupted run's losses."""
    folder = str(tmp_path / "ck")
    saved = spawn(functools.partial(_ckpt_body, folder, "save", optimizer), world=4)
    loaded = spawn(functools.partial(_ckpt_body, folder, "load", optimizer), world=4)
    for out in (saved, loaded):
        for r in out.values():
            assert r[0] == "ok", r[1]
    a, b = torch.tensor(saved[0][1]), torch.tensor(loaded[0][1])
    assert torch.allclose(a, b, rtol=1e-4, atol=1e-4), (a, b)
