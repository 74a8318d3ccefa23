"""FSDP x TP (2-D mesh) training on CPU with gloo: the Llama TP plan
(column/row-parallel attention and MLP) on a 2 x 2 (dp_shard, tp) mesh must
reproduce the data-parallel-only run on the same global batch for Muon and
Dion2 (whose TP paths assemble whole matrices before Newton-Schulz), and
train without error for AdamW and Dion."""
import functools

import pytest
import torch

from test_distributed_cpu import spawn


def _train_body(optimizer, dp_shard, tp, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64),
                        seq_len=32, local_batch_size=2, steps=4, warmup_steps=0, dp_shard=dp_shard, tp=tp,
                        optimizer=opt, seed=5)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    losses = []
    for _ in range(4):
        t, l = tr.data.next()
        losses.append(float(tr.train_step(t, l)))
    return losses


def _train(optimizer, dp_shard, tp):
    return functools.partial(_train_body, optimizer, dp_shard, tp)


@pytest.mark.parametrize("optimizer", ["Muon", "Dion2"])
def test_fsdp_tp_matches_dp(optimizer):
    ref = spawn(_train(optimizer, 2, 1), world=2)
    got = spawn(_train(optimizer, 2, 2), world=4)
    for r in ref.values():
        assert r[0] == "ok", r[1]
    for r in got.values():
        assert r[0] == "ok", r[1]
    a = torch.tensor(ref[0][1])
    b = torch.tensor(got[0][1])
    assert torch.isfinite(b).all()
    assert torch.allclose(a, b, rtol=2e-3, atol=2e-3), (a, b)


@pytest.mark.parametrize("optimizer", ["AdamW", "Dion", "AdaDionV2"])
def test_fsdp_tp_trains(optimizer):
    got = spawn(_train(optimizer, 2, 2), world=4)
    for r in got.values():
        assert r[0] == "ok", r[1]
    b = torch.tensor(got[0][1])
    assert torch.isfinite(b).all()


def _ckpt_body(folder, phase, optimizer, dp_shard, tp, rank, world):
    from dion_b200.checkpoint import CheckpointManager
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=64),
                        seq_len=32, local_batch_size=4 // dp_shard, steps=4, warmup_steps=0, dp_shard=dp_shard, tp=tp,
                        optimizer=opt, seed=5)
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
    import torch.distributed as dist

    out = []
    for _ in range(2):
        loss = tr.train_step(*tr.data.next()).detach().clone()
        if dp_shard > 1:  # mean over the data-parallel ranks (TP ranks hold the same value)
            dist.all_reduce(loss)
            loss /= world
        out.append(float(loss))
    return out


# Dion keeps Q on the side its sharding dictates (the FSDP x TP layout
# orients column-parallel matrices differently from one process); loading a
# checkpoint into a layout that flips a matrix converts its Q to the other
# side (column-normalised M Q), so the resumed run follows the 2-D run.
@pytest.mark.parametrize("optimizer,load_layout", [("Muon", (1, 1)), ("Dion", (2, 2)), ("Dion", (1, 1))])
def test_fsdp_tp_checkpoint_resume(tmp_path, optimizer, load_layout):
    """A checkpoint of the FSDP 2 x TP 2 layout resumes (parameters and
    optimizer state resharded by DCP) and continues with the losses of the
    uninterrupted 2-D run."""
    folder = str(tmp_path / "ck")
    saved = spawn(functools.partial(_ckpt_body, folder, "save", optimizer, 2, 2), world=4)
    for r in saved.values():
        assert r[0] == "ok", r[1]
    dp, tp = load_layout
    loaded = spawn(functools.partial(_ckpt_body, folder, "load", optimizer, dp, tp), world=dp * tp)
    assert loaded[0][0] == "ok", loaded[0][1]
    a, b = torch.tensor(saved[0][1]), torch.tensor(loaded[0][1])
    assert torch.allclose(a, b, rtol=2e-3, atol=2e-3), (a, b)


def _lowrank_tp_body(rank, world):
    try:
        _train_body("SDion", 1, 2, rank, world)
    except ValueError as e:
        return [str(e)]
    return ["no error"]


def test_adadion_family_rejects_tensor_parallelism():
    out = spawn(_lowrank_tp_body, world=2)
    for r in out.values():
        assert r[0] == "ok", r[1]
        assert "tensor-parallel" in r[1][0], r[1]
