"""Pipeline parallelism on CPU (gloo): a 2-stage pipeline (1F1B and GPipe,
alone and with FSDP over 2 data-parallel ranks) reproduces the losses of the
unpipelined run on the same data."""
import functools
import os

import pytest
import torch

from test_distributed_cpu import spawn


def _body(pp, dp, schedule, optimizer, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=4, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=4, steps=3, warmup_steps=0, dp_shard=dp, pp=pp, pp_schedule=schedule,
                        pp_microbatches=2, optimizer=opt, seed=7, use_fsdp=dp > 1)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    out = []
    for _ in range(3):
        t, l = tr.data.next()
        out.append(float(tr.train_step(t, l)))
    return out


def _run(pp, dp, schedule="1F1B", optimizer="Muon"):
    world = pp * dp
    res = spawn(functools.partial(_body, pp, dp, schedule, optimizer), world=world)
    for r in res.values():
        assert r[0] == "ok", r[1]
    return torch.tensor(res[0][1]), res


@pytest.mark.parametrize("schedule", ["1F1B", "GPipe"])
def test_pipeline_matches_single(schedule):
    ref, _ = _run(1, 1)
    got, res = _run(2, 1, schedule)
    assert torch.allclose(ref, got, rtol=2e-3, atol=2e-3), (ref, got)
    assert torch.equal(torch.tensor(res[1][1]), got)  # every stage reports the same loss


def test_pipeline_with_fsdp():
    ref, _ = _run(1, 2)
    got, _ = _run(2, 2)
    assert torch.allclose(ref, got, rtol=2e-3, atol=2e-3), (ref, got)


def _ckpt_body(folder, phase, pp, rank, world):
    """phase "save": 2 steps, checkpoint, 2 more steps; "load": resume, 2 steps."""
    from dion_b200.checkpoint import CheckpointManager
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    opt = HybridOptimizersContainer.Config(name="Muon", lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=4, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=4, steps=4, warmup_steps=0, dp_shard=1, pp=pp, pp_microbatches=2,
                        optimizer=opt, seed=7, use_fsdp=False)
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
    return [float(tr.train_step(*tr.data.next())) for _ in range(2)]


def test_pipeline_checkpoint_resumes_without_pipeline(tmp_path):
    """Stages keep the full model's parameter names, so a checkpoint written by
    a 2-stage pipeline loads into the unpipelined model (and optimizer) and
    continues with the pipeline's losses."""
    folder = str(tmp_path / "ck")
    saved = spawn(functools.partial(_ckpt_body, folder, "save", 2), world=2)
    for r in saved.values():
        assert r[0] == "ok", r[1]
    loaded = spawn(functools.partial(_ckpt_body, folder, "load", 1), world=1)
    assert loaded[0][0] == "ok", loaded[0][1]
    a, b = torch.tensor(saved[0][1]), torch.tensor(loaded[0][1])
    assert torch.allclose(a, b, rtol=2e-3, atol=2e-3), (a, b)


def _no_fsdp_dp_body(rank, world):
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    try:
        Trainer(TrainerConfig(model="tiny", seq_len=16, local_batch_size=2, steps=1, pp=1, use_fsdp=False),
                device=torch.device("cpu"))
    except ValueError as e:
        return [str(e)]
    return ["no error"]


def test_data_parallel_without_fsdp_is_rejected():
    """Two data-parallel ranks with use_fsdp=False would train unsynchronised
    replicas; the trainer refuses the layout."""
    out = spawn(_no_fsdp_dp_body, world=2)
    for r in out.values():
        assert r[0] == "ok", r[1]
        assert "dp_replicate" in r[1][0], r[1]


def _val_body(folder, pp, rank, world):
    from dion_b200.data import write_token_file
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    val = os.path.join(folder, "val.bin")
    if rank == 0 and not os.path.exists(val):
        write_token_file(val, torch.randint(0, 512, (4000,), generator=torch.Generator().manual_seed(3)))
    import torch.distributed as dist

    dist.barrier()
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=4, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=4, steps=1, warmup_steps=0, dp_shard=1, pp=pp, pp_microbatches=2,
                        optimizer=HybridOptimizersContainer.Config(name="Muon"), seed=7, use_fsdp=False,
                        val_dataset=val)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    return [tr.validate(2)]


def test_pipeline_validation_matches_unpipelined(tmp_path):
    """Validation through the pipeline's forward-only schedule gives the
    unpipelined model's loss, on every stage."""

    one = spawn(functools.partial(_val_body, str(tmp_path), 1), world=1)
    two = spawn(functools.partial(_val_body, str(tmp_path), 2), world=2)
    for out in (one, two):
        for r in out.values():
            assert r[0] == "ok", r[1]
    assert two[0][1] == two[1][1]
    assert abs(one[0][1][0] - two[0][1][0]) < 1e-4, (one[0][1], two[0][1])
