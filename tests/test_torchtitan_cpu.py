"""The torchtitan integration: the registered train spec builds this
package's optimizer container for torchtitan's Llama model, torchtitan's LR
scheduler drives it, and a step trains (single process, CPU)."""
import pytest
import torch

tt = pytest.importorskip("torchtitan")


def test_train_spec_builds_and_steps():
    from torchtitan.components.lr_scheduler import build_lr_schedulers
    from torchtitan.config.job_config import LRScheduler, Optimizer
    from torchtitan.models.llama3 import llama3_configs
    from torchtitan.models.llama3.model.model import Transformer
    from torchtitan.protocols.train_spec import get_train_spec

    from dion_b200.integration import torchtitan_shim as shim

    assert shim.register()
    spec = get_train_spec(shim.TRAIN_SPEC_NAME)
    assert spec.build_optimizers_fn is shim.build_dion_optimizers
    args = llama3_configs["debugmodel"]
    torch.manual_seed(0)
    model = Transformer(args)
    model.init_weights()
    oc = Optimizer(name="Dion", lr=0.02, weight_decay=0.01)
    oc.rank_fraction = 0.5
    dims = type("PD", (), {"world_size": 1})()
    opts = spec.build_optimizers_fn([model], oc, dims)
    inner = opts.optimizers[0]
    assert type(inner).__name__ == "Dion"
    assert any(g.get("algorithm") == "adamw" for g in inner.param_groups)
    scheds = build_lr_schedulers(opts, LRScheduler(warmup_steps=2), 10)
    tok = torch.randint(0, args.vocab_size, (2, 32))
    losses = []
    for _ in range(3):
        out = model(tok)
        loss = torch.nn.functional.cross_entropy(out[:, :-1].flatten(0, 1).float(), tok[:, 1:].flatten())
        loss.backward()
        opts.step()
        scheds.step()
        opts.zero_grad()
        losses.append(float(loss.detach()))
    assert all(l == l for l in losses) and losses[-1] < losses[0]
    sd = opts.state_dict()
    assert any(k.startswith("state.") and k.endswith(".momentum") for k in sd)


def test_extension_fields_merge_into_optimizer_section():
    from torchtitan.config.manager import ConfigManager

    from dion_b200.integration import torchtitan_shim as shim

    merged = ConfigManager._merge_configs(__import__("torchtitan.config.job_config", fromlist=["JobConfig"]).JobConfig,
                                          shim.JobConfig)
    job = merged()
    assert job.optimizer.rank_fraction == 0.25 and job.optimizer.lr > 0
