"""Edge-case matrix over every optimizer (CPU), after the reference's
pre-push suite (ada_dion/tests/test_adadion_prepush.py: dtypes, shapes down
to 1 x 1, state-dict round trip, edge cases, long runs, simulated FSDP
shards): each optimizer must keep parameters finite and in their dtype on
fp32 / bf16 / fp16 matrices of degenerate shapes, skip parameters without a
gradient, survive zero gradients, and resume from its state dict to the
same parameters as an uninterrupted run."""
import copy

import pytest
import torch
import torch.nn as nn

from dion_b200.optim import AGDion, AdaDion, AdaDionV2, Dion, Dion2, GSDion, Muon, QCDion, SDion

LOWRANK = dict(lr=0.02, init_rank=4, rank_min=1, rank_max=16)
ALL = [
    (Muon, dict(lr=0.02)),
    (Dion, dict(lr=0.02, rank_fraction=0.5)),
    (Dion2, dict(lr=0.02, fraction=0.5)),
    (AdaDionV2, dict(lr=0.02, adaptive_rank=True, init_rank_fraction=0.5, rank_min=1)),
    (AdaDion, LOWRANK),
    (SDion, LOWRANK),
    (GSDion, LOWRANK),
    (AGDion, LOWRANK),
    (QCDion, LOWRANK),
]
IDS = [c.__name__ for c, _ in ALL]
SHAPES = [(1, 1), (1, 8), (8, 1), (2, 3), (17, 5), (5, 17), (16, 16)]


def _step(opt, params, seed):
    g = torch.Generator().manual_seed(seed)
    for p in params:
        p.grad = torch.randn(p.shape, generator=g).to(p.dtype)
    opt.step()


@pytest.mark.parametrize("cls,kw", ALL, ids=IDS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dtypes_and_degenerate_shapes(cls, kw, dtype):
    torch.manual_seed(0)
    params = [nn.Parameter(torch.randn(s).to(dtype)) for s in SHAPES]
    before = [p.detach().clone() for p in params]
    opt = cls(params, **kw)
    for i in range(3):
        _step(opt, params, i)
    for p, b, s in zip(params, before, SHAPES):
        assert p.dtype == dtype and tuple(p.shape) == s
        assert torch.isfinite(p.float()).all(), (s, p)
        assert not torch.equal(p, b), s


@pytest.mark.parametrize("cls,kw", ALL, ids=IDS)
def test_params_without_grad_are_skipped_and_zero_grad_is_finite(cls, kw):
    torch.manual_seed(1)
    a, b = nn.Parameter(torch.randn(12, 8)), nn.Parameter(torch.randn(12, 8))
    opt = cls([a, b], **kw)
    b0 = b.detach().clone()
    a.grad = torch.randn_like(a)
    opt.step()  # b has no gradient
    assert torch.equal(b, b0)
    a.grad = torch.zeros_like(a)
    b.grad = torch.zeros_like(b)
    opt.step()
    assert torch.isfinite(a).all() and torch.isfinite(b).all()


@pytest.mark.parametrize("cls,kw", ALL, ids=IDS)
def test_resume_from_state_dict_matches_uninterrupted(cls, kw):
    torch.manual_seed(2)
    init = [torch.randn(24, 16), torch.randn(16, 24), torch.randn(20, 20)]
    ref = [nn.Parameter(t.clone()) for t in init]
    ropt = cls(ref, **kw)
    for i in range(6):
        _step(ropt, ref, i)

    first = [nn.Parameter(t.clone()) for t in init]
    fopt = cls(first, **kw)
    for i in range(3):
        _step(fopt, first, i)
    sd = copy.deepcopy(fopt.state_dict())
    resumed = [nn.Parameter(p.detach().clone()) for p in first]
    opt = cls(resumed, **kw)
    opt.load_state_dict(sd)
    for i in range(3, 6):
        _step(opt, resumed, i)
    for a, b in zip(resumed, ref):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("cls,kw", ALL, ids=IDS)
def test_long_run_stays_finite_and_bounded(cls, kw):
    """200 steps on noisy gradients of a quadratic: parameters stay finite
    and the loss ends below where it started."""
    torch.manual_seed(3)
    p = nn.Parameter(torch.randn(32, 24))
    opt = cls([p], **kw)
    start = float((p.detach() ** 2).sum())
    g = torch.Generator().manual_seed(4)
    for _ in range(200):
        p.grad = 2 * p.detach() + 0.1 * torch.randn(p.shape, generator=g)
        opt.step()
    assert torch.isfinite(p).all()
    assert float((p.detach() ** 2).sum()) < start


@pytest.mark.parametrize("cls,kw", ALL, ids=IDS)
def test_mixed_groups_route_scalars_to_adamw_and_lion(cls, kw):
    torch.manual_seed(5)
    w = nn.Parameter(torch.randn(16, 8))
    bias = nn.Parameter(torch.randn(16))
    norm = nn.Parameter(torch.ones(8))
    opt = cls([{"params": [w]},
               {"params": [bias], "algorithm": "adamw", "lr": 1e-2},
               {"params": [norm], "algorithm": "lion", "lr": 1e-3}], **kw)
    b0, n0 = bias.detach().clone(), norm.detach().clone()
    for i in range(2):
        _step(opt, [w, bias, norm], i)
    assert not torch.equal(bias, b0) and not torch.equal(norm, n0)
    # Lion's sign update moves each coordinate by at most lr per step (plus decoupled decay)
    assert float((norm - n0).detach().abs().max()) <= 2 * 1e-3 * 1.1


def _state_bytes(opt):
    n = 0
    for st in opt.state.values():
        for v in st.values():
            if isinstance(v, torch.Tensor):
                n += v.numel() * v.element_size()
    return n


@pytest.mark.parametrize("cls,kw", ALL, ids=IDS)
def test_state_does_not_grow_over_steps(cls, kw):
    """Stress check: after warm-up the optimizer state (and the optimizer's
    own caches) stay the same size however many steps run."""
    torch.manual_seed(6)
    params = [nn.Parameter(torch.randn(s)) for s in [(32, 16), (16, 32), (24, 24), (24, 24)]]
    opt = cls(params, **kw)
    for i in range(12):
        _step(opt, params, i)
    size = _state_bytes(opt)
    caches = {k: len(v) for k, v in vars(opt).items() if isinstance(v, (dict, list)) and k != "param_groups"}
    for i in range(12, 60):
        _step(opt, params, i)
    assert _state_bytes(opt) <= size
    later = {k: len(v) for k, v in vars(opt).items() if isinstance(v, (dict, list)) and k != "param_groups"}
    assert later == caches, (caches, later)


GUARDED = [(c, kw) for c, kw in ALL if c not in (Muon, Dion2)]


@pytest.mark.parametrize("cls,kw", GUARDED, ids=[c.__name__ for c, _ in GUARDED])
def test_nan_gradient_does_not_reach_the_weights(cls, kw):
    """The Dion family guards its low-rank update against NaN / Inf (the
    reference's fix_all_zero_or_nan and NaN zeroing; GSDion also skips a
    non-finite step scale). Muon and Dion2 have no such guard, like the
    reference's Muon: a NaN gradient reaches their weights."""
    torch.manual_seed(7)
    p = nn.Parameter(torch.randn(16, 8))
    opt = cls([p], **kw)
    g = torch.randn(16, 8)
    g[3, 2] = float("nan")
    p.grad = g
    opt.step()
    assert torch.isfinite(p).all()
