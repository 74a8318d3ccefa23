"""Pipeline parallelism on CPU (gloo): a 2-stage pipeline (1F1B and GPipe,
alone and with FSDP over 2 data-parallel ranks) reproduces the losses of the
unpipelined run on the same data."""
import functools

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
