"""Dion2, AdaDion, AdaDionV2 (adaptive) and the research variants on CPU:
invariants, convergence, state keys, diagnostics and checkpoint round trip
(mirrors the reference's per-optimizer unit tests)."""
import copy

import pytest
import torch
import torch.nn as nn

from dion_b200.optim import AGDion, AdaDion, AdaDionV2, Dion2, GSDion, QCDion, SDion

VARIANTS = [
    (AdaDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32, warmup_rank=16)),
    (SDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32)),
    (GSDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32, warmup_rank=16)),
    (AGDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32)),
    (QCDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32)),
    (Dion2, dict(lr=0.02, fraction=0.25, ef_decay=0.95)),
    (AdaDionV2, dict(lr=0.02, adaptive_rank=True, init_rank_fraction=0.25, rank_min=4)),
]
IDS = [c.__name__ for c, _ in VARIANTS]


@pytest.mark.parametrize("cls,kw", VARIANTS, ids=IDS)
@pytest.mark.parametrize("shape", [(32, 16), (16, 48)])
def test_step_finite_and_changes(cls, kw, shape):
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(shape))
    before = p.detach().clone()
    opt = cls([p], **kw)
    for _ in range(3):
        p.grad = torch.randn_like(p) * 0.1
        opt.step()
    assert torch.isfinite(p).all()
    assert not torch.equal(p.detach(), before)


@pytest.mark.parametrize("cls,kw", VARIANTS, ids=IDS)
def test_weight_decay_shrinks(cls, kw):
    p = nn.Parameter(torch.ones(32, 64))
    opt = cls([p], **dict(kw, weight_decay=0.5))
    n0 = p.norm().item()
    p.grad = torch.zeros_like(p)
    opt.step()
    assert torch.isfinite(p).all()
    assert p.norm().item() < n0


@pytest.mark.parametrize("cls,kw", VARIANTS, ids=IDS)
def test_quadratic_loss_decreases(cls, kw):
    torch.manual_seed(42)
    p = nn.Parameter(torch.randn(32, 64))
    opt = cls([p], **kw)
    losses = []
    for _ in range(60):
        opt.zero_grad()
        loss = (p**2).sum()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("frac", [0.1, 0.25, 0.5, 0.75, 1.0])
def test_dion2_fractions(frac):
    p = nn.Parameter(torch.randn(40, 80))
    opt = Dion2([p], lr=0.02, fraction=frac)
    p.grad = torch.randn_like(p) * 0.01
    opt.step()
    assert not torch.isnan(p).any()


def test_dion2_selective_decay_and_random():
    torch.manual_seed(0)
    p = nn.Parameter(torch.zeros(8, 16))
    opt = Dion2([p], lr=0.0, fraction=0.25, ef_decay=0.5, weight_decay=0.0)
    g = torch.zeros(8, 16)
    g[3] = 10.0
    g[6] = 5.0
    g[0] = 0.1
    p.grad = g.clone()
    opt.step()
    M = opt.state[p]["momentum"]
    # the two largest-L1 rows were used and decayed, the others kept whole
    torch.testing.assert_close(M[3], torch.full((16,), 5.0))
    torch.testing.assert_close(M[6], torch.full((16,), 2.5))
    torch.testing.assert_close(M[0], torch.full((16,), 0.1))
    p2 = nn.Parameter(torch.randn(8, 16))
    opt2 = Dion2([p2], lr=0.02, fraction=0.5, selection_method="random")
    p2.grad = torch.randn_like(p2)
    opt2.step()
    assert torch.isfinite(p2).all()


def test_adadion_state_keys_and_diagnostics():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(64, 32))
    b = nn.Parameter(torch.randn(32))
    opt = AdaDion([{"params": [p]}, {"params": [b], "algorithm": "adamw", "lr": 1e-3}], lr=0.02, init_rank=8,
                  rank_min=4, rank_max=32, rank_warmup_steps=2, warmup_rank=16, anchor_period=3)
    for _ in range(6):
        p.grad = torch.randn_like(p)
        b.grad = torch.randn_like(b)
        opt.step()
    st = opt.state[p]
    assert {"M", "Qbuf", "r", "tr", "erank_ema", "aerr_ema", "Q_anchor", "step"} <= set(st)
    assert set(opt.state[b]) == {"step", "m1", "m2"}
    assert opt.get_rank() and opt.get_effective_rank() and opt.get_aerr()
    assert "param_0" in opt.get_anchor_drift()


def test_adadion_state_dict_roundtrip_and_ws_stamp():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(32, 32))
    opt = AdaDion([p], lr=0.02, init_rank=8, rank_min=4, rank_max=16)
    p.grad = torch.randn_like(p)
    opt.step()
    sd = copy.deepcopy(opt.state_dict())
    p2 = nn.Parameter(p.detach().clone())
    opt2 = AdaDion([p2], lr=0.02, init_rank=8, rank_min=4, rank_max=16)
    opt2.load_state_dict(sd)
    torch.testing.assert_close(opt2.state[p2]["M"], opt.state[p]["M"])
    sd["_adadion_ws"] = 4
    with pytest.raises(RuntimeError):
        opt2.load_state_dict(sd)


def test_sdion_modes_counted():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(32, 32))
    opt = SDion([p], lr=0.01, init_rank=8, rank_min=4, rank_max=16, tau_drift_safe=10.0, tau_tail_recovery=10.0)
    for _ in range(8):
        p.grad = torch.randn_like(p) * 0.01
        opt.step()
    c = opt.get_mode_counts()
    assert c["total"] == 8 and c["skip"] > 0
    assert "p0/mode" in opt.get_diagnostics()


def test_adadion_v2_adaptive_rank_moves():
    torch.manual_seed(0)
    ps = [nn.Parameter(torch.randn(64, 64)) for _ in range(3)]
    opt = AdaDionV2(ps, lr=0.01, adaptive_rank=True, init_rank_fraction=0.125, rank_fraction_max=0.5,
                    rank_min=4, rank_quantize=4, rank_step_up=8, rank_step_down=4)
    for _ in range(5):
        for p in ps:
            p.grad = torch.randn_like(p)
        opt.step()
    ranks = opt.get_rank()
    assert len(ranks) == 3
    st = opt.state[ps[0]]
    assert {"momentum", "Q", "r", "r_cap", "transpose", "erank_ema", "aerr_ema", "ada_step"} <= set(st)
    assert st["r_cap"] == 32 and st["ada_step"] == 5
    assert all(v is not None for v in opt.get_effective_rank().values())
    assert all(torch.isfinite(p).all() for p in ps)


def test_adadion_v2_matches_dion_when_not_adaptive():
    from dion_b200.optim import Dion

    torch.manual_seed(3)
    X = torch.randn(48, 32)
    G = torch.randn(48, 32)
    a = nn.Parameter(X.clone())
    b = nn.Parameter(X.clone())
    o1 = AdaDionV2([a], lr=0.02, rank_fraction_max=0.5)
    torch.manual_seed(7)
    a.grad = G.clone()
    o1.step()
    o2 = Dion([b], lr=0.02, rank_fraction=0.5, weight_decay=0.1)
    torch.manual_seed(7)
    b.grad = G.clone()
    o2.step()
    torch.testing.assert_close(a.detach(), b.detach())
