"""Checkpoints move between this package and the reference implementation.

Optimizer state written by the reference's optimizers (``dion.Muon`` and
``ada_dion.optim.adadion_v2.AdaDionV2``, installed in baseline/_ref) through
DCP with flattened keys (the container's format,
ada_dion/integration/hybrid_optimizer.py:288-307) loads into this package's
Muon / Dion, and the reverse. After loading, both implementations take the
same next step: Muon has no random draws, and Dion's orthonormalised P is
unique up to column signs whatever sketch produced it, so the two updates
agree to rounding.
"""
import os
import sys

import pytest
import torch
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.state_dict import (StateDictOptions, get_optimizer_state_dict,
                                                     set_optimizer_state_dict)

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "ada_dion")),
                                reason="reference not installed in baseline/_ref")
FLAT = StateDictOptions(flatten_optimizer_state_dict=True)


@pytest.fixture(autouse=True)
def _eager_reference():
    """Run the reference's torch.compile'd helpers eagerly (no C++ toolchain needed)."""
    import torch._dynamo

    old = torch._dynamo.config.disable
    torch._dynamo.config.disable = True
    if REF not in sys.path:
        sys.path.insert(0, REF)
    yield
    torch._dynamo.config.disable = old


def _model(seed=0):
    from dion_b200.models.llama3 import Transformer, llama3_config

    torch.manual_seed(seed)
    m = Transformer(llama3_config("tiny", n_layers=2, vocab_size=512, max_seq_len=32))
    m.init_weights()
    return m


def _groups(model):
    from dion_b200.integration.param_grouper import group_params_for_hybrid

    g = group_params_for_hybrid(model)
    mats = {id(p) for p in g.matrix_params}
    scalar = dict(algorithm="adamw", lr=3e-4, beta1=0.9, beta2=0.95, epsilon=1e-8, weight_decay=0.1)
    return [{"params": [p for p in model.parameters() if id(p) in mats]},
            {"params": [p for p in model.parameters() if id(p) not in mats], **scalar}]


def _make(impl, kind, model):
    if impl == "ours":
        from dion_b200.optim import Dion, Muon

        if kind == "muon":
            return Muon(_groups(model), lr=0.02, mu=0.95, weight_decay=0.01)
        return Dion(_groups(model), lr=0.02, mu=0.95, rank_fraction=0.25, weight_decay=0.01)
    if kind == "muon":
        from dion import Muon as RefMuon

        return RefMuon(_groups(model), fsdp_mesh_dim=0, world_mesh=None, lr=0.02, mu=0.95, weight_decay=0.01)
    from ada_dion.optim.adadion_v2 import AdaDionV2

    return AdaDionV2(_groups(model), lr=0.02, mu=0.95, rank_fraction_max=0.25, weight_decay=0.01)


def _grads(model, step):
    g = torch.Generator().manual_seed(1000 + step)
    for p in model.parameters():
        p.grad = torch.randn(p.shape, generator=g) * 0.1


def _train(opt, model, steps, start=0):
    for s in range(start, start + steps):
        _grads(model, s)
        opt.step()
        opt.zero_grad(set_to_none=True)


@pytest.mark.parametrize("kind", ["muon", "dion"])
@pytest.mark.parametrize("src,dst", [("reference", "ours"), ("ours", "reference")])
def test_optimizer_checkpoint_crosses_implementations(tmp_path, kind, src, dst):
    m_src = _model()
    o_src = _make(src, kind, m_src)
    _train(o_src, m_src, 3)
    dcp.save({"model": m_src.state_dict(), "optimizer": get_optimizer_state_dict(m_src, o_src, options=FLAT)},
             checkpoint_id=str(tmp_path / "ckpt"))

    m_dst = _model(seed=7)  # different weights: everything must come from the checkpoint
    o_dst = _make(dst, kind, m_dst)
    sd = {"model": m_dst.state_dict(), "optimizer": get_optimizer_state_dict(m_dst, o_dst, options=FLAT)}
    dcp.load(sd, checkpoint_id=str(tmp_path / "ckpt"))
    m_dst.load_state_dict(sd["model"])
    set_optimizer_state_dict(m_dst, o_dst, sd["optimizer"], options=FLAT)

    names_src = dict(m_src.named_parameters())
    for name, p in m_dst.named_parameters():
        a, b = o_src.state[names_src[name]], o_dst.state[p]
        assert set(a) == set(b), name
        for key in a:
            if torch.is_tensor(a[key]):
                torch.testing.assert_close(b[key].float(), a[key].float(), rtol=0, atol=0, msg=f"{name}.{key}")
    assert [g["step"] for g in o_dst.param_groups] == [g["step"] for g in o_src.param_groups]

    # the next step from the loaded state matches the source implementation's next step
    before = {k: v.detach().clone() for k, v in m_dst.state_dict().items()}
    _train(o_src, m_src, 1, start=3)
    _train(o_dst, m_dst, 1, start=3)
    for name, p in m_dst.named_parameters():
        q = names_src[name]
        upd = (q.detach() - before[name]).norm()
        if upd > 0:
            rel = ((p.detach() - q.detach()).norm() / upd).item()
            assert rel < 2e-2, (name, rel)
