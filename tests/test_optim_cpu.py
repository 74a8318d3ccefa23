"""Optimizer unit tests on CPU (reference test strategy: single-step
invariants, weight decay, rank fractions, convergence on a quadratic, state
keys) plus one-step comparisons against the float64 oracle."""
import math

import pytest
import torch

from dion_b200 import ops
from dion_b200.optim import Dion, Muon, oracle


def _quad_loss_decreases(opt_factory, steps=60):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(32, 48) * 0.5)
    opt = opt_factory([p])
    first = None
    for _ in range(steps):
        opt.zero_grad()
        loss = (p**2).sum()
        loss.backward()
        opt.step()
        first = first if first is not None else loss.item()
    return first, (p**2).sum().item()


@pytest.mark.parametrize("cls,kw", [(Muon, dict(lr=0.02)), (Dion, dict(lr=0.02, rank_fraction=0.5))])
def test_single_step_finite_and_changes(cls, kw):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(64, 32))
    before = p.detach().clone()
    opt = cls([p], **kw)
    p.grad = torch.randn_like(p)
    opt.step()
    assert torch.isfinite(p).all()
    assert not torch.equal(before, p.detach())


@pytest.mark.parametrize("cls,kw", [(Muon, dict(lr=0.02, weight_decay=0.5)),
                                    (Dion, dict(lr=0.02, weight_decay=0.5, rank_fraction=0.25))])
def test_weight_decay_shrinks(cls, kw):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(32, 32))
    n0 = p.norm().item()
    opt = cls([p], **kw)
    for _ in range(5):
        p.grad = torch.zeros_like(p)
        opt.step()
    assert p.norm().item() < n0


@pytest.mark.parametrize("rf", [0.1, 0.25, 0.5, 1.0])
def test_dion_rank_fractions(rf):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(40, 24))
    opt = Dion([p], lr=0.01, rank_fraction=rf)
    p.grad = torch.randn_like(p)
    opt.step()
    st = opt.state[p]
    r = min(int(math.ceil(rf * 24)), 24)
    assert st["Q"].shape == (24, r)
    assert set(st.keys()) == {"momentum", "Q"}
    assert torch.isfinite(p).all()


@pytest.mark.parametrize("cls,kw", [(Muon, dict(lr=0.05)), (Dion, dict(lr=0.05, rank_fraction=0.5))])
def test_quadratic_convergence(cls, kw):
    first, last = _quad_loss_decreases(lambda ps: cls(ps, **kw))
    assert last < first


def test_muon_matches_oracle():
    torch.manual_seed(1)
    for shape in [(48, 32), (24, 40)]:
        X = torch.randn(shape)
        G = torch.randn(shape)
        p = torch.nn.Parameter(X.clone())
        opt = Muon([p], lr=0.02, mu=0.9, weight_decay=0.1, nesterov=True, ns_coeffs="keller")
        p.grad = G.clone()
        opt.step()
        Xr, Mr = oracle.muon_step(X, G, torch.zeros(shape), 0.02, 0.9, 0.1, True, ops.KELLER_NS_COEFFS)
        # bf16 Newton-Schulz input vs float64 oracle
        assert (p.detach().double() - Xr).norm() / (Xr - X.double()).norm() < 0.05
        torch.testing.assert_close(opt.state[p]["momentum"].double(), Mr, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("shape", [(48, 32), (32, 48), (40, 40)])
def test_dion_matches_oracle(shape):
    torch.manual_seed(2)
    X = torch.randn(shape)
    G = torch.randn(shape)
    p = torch.nn.Parameter(X.clone())
    opt = Dion([p], lr=0.02, mu=0.9, weight_decay=0.1, rank_fraction=0.5)
    p.grad = G.clone()
    # capture the initial Q the optimizer draws
    opt._get_or_initialize_state(p, opt.param_groups[0])
    Q0 = opt.state[p]["Q"].clone()
    opt.step()
    Xr, Mr, Qr = oracle.dion_step(X, G, torch.zeros(shape), Q0, 0.02, 0.9, 0.1)
    torch.testing.assert_close(p.detach().double(), Xr, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(opt.state[p]["momentum"].double(), Mr, rtol=1e-4, atol=1e-4)
    # Q columns agree up to sign
    Qn = opt.state[p]["Q"].double()
    torch.testing.assert_close(Qn.abs(), Qr.abs(), rtol=1e-4, atol=1e-4)


def test_dion_zero_gradient_guard():
    p = torch.nn.Parameter(torch.randn(16, 8))
    opt = Dion([p], lr=0.01, weight_decay=0.0, rank_fraction=0.5)
    p.grad = torch.zeros_like(p)
    before = p.detach().clone()
    opt.step()
    assert torch.isfinite(p).all()
    torch.testing.assert_close(p.detach(), before)


def test_scalar_algorithms_route():
    torch.manual_seed(0)
    w = torch.nn.Parameter(torch.randn(16, 16))
    b = torch.nn.Parameter(torch.randn(16))
    e = torch.nn.Parameter(torch.randn(10, 16))
    opt = Dion([{"params": [w]}, {"params": [b], "algorithm": "adamw"}, {"params": [e], "algorithm": "lion"}],
               lr=0.01, rank_fraction=0.5)
    for t in (w, b, e):
        t.grad = torch.randn_like(t)
    opt.step()
    assert set(opt.state[b].keys()) == {"momentum", "variance"}
    assert set(opt.state[e].keys()) == {"momentum"}


def test_philox_known_answers_and_statistics():
    """Integer stage against the published Philox-4x32-10 known-answer vectors
    (Random123 kat_vectors); the normals have mean 0 / std 1 and depend only
    on (key, stream, index)."""
    from dion_b200.ops import _MASK32, _PHILOX_M, _PHILOX_W, philox_normal

    def philox(ctr, key):
        c = [torch.tensor([v], dtype=torch.int64) for v in ctr]
        k0, k1 = key
        for _ in range(10):
            p0, p1 = _PHILOX_M[0] * c[0], _PHILOX_M[1] * c[2]
            c = [((p1 >> 32) & _MASK32) ^ c[1] ^ k0, p1 & _MASK32, ((p0 >> 32) & _MASK32) ^ c[3] ^ k1, p0 & _MASK32]
            k0, k1 = (k0 + _PHILOX_W[0]) & _MASK32, (k1 + _PHILOX_W[1]) & _MASK32
        return [int(x) for x in c]

    assert philox([0, 0, 0, 0], (0, 0)) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    m = 0xFFFFFFFF
    assert philox([m, m, m, m], (m, m)) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], (0xA4093822, 0x299F31D0)) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    x = philox_normal((200, 500), 123, 9, 1.0, "cpu")
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
    assert torch.equal(x, philox_normal((200, 500), 123, 9, 1.0, "cpu"))
    assert not torch.equal(x, philox_normal((200, 500), 123, 10, 1.0, "cpu"))
    # element i does not depend on the requested size
    assert torch.equal(philox_normal((7,), 5, 1, 2.0, "cpu"), philox_normal((10,), 5, 1, 2.0, "cpu")[:7])


def test_stream_pool_is_inactive_without_cuda_or_with_one_unit():
    """Side streams only for several units on a CUDA device; otherwise use() is a no-op."""
    from dion_b200.optim._utils import StreamPool

    pool = StreamPool(3)
    for dev, units in ((torch.device("cpu"), 4), (torch.device("cpu"), 1)):
        s = pool.session(dev, units)
        assert not s.active
        with s.use(0):
            pass
        s.join()
    assert not StreamPool(3, enabled=False).session(torch.device("cuda", 0), 4).active


def test_device_list_is_cached_by_value():
    from dion_b200.optim._utils import device_list

    a = device_list([3, 1, 2], torch.int64, torch.device("cpu"))
    b = device_list([3, 1, 2], torch.int64, torch.device("cpu"))
    c = device_list([3, 1, 4], torch.int64, torch.device("cpu"))
    assert a is b and a.tolist() == [3, 1, 2] and c.tolist() == [3, 1, 4]
    assert device_list((1, 2), torch.int32, "cpu").dtype == torch.int32


def test_muon_side_stream_size_classes():
    """Groups whose Newton-Schulz GEMMs fill the GPU stay on the main stream."""
    params = [torch.nn.Parameter(torch.zeros(512, 2048)) for _ in range(4)]
    opt = Muon(params, lr=0.02)
    assert opt._ns_tiles(params) == 4 * 2 * 8  # 4 matrices x (512/256) x (2048/256) tiles
    big = [torch.nn.Parameter(torch.zeros(4096, 4096)) for _ in range(8)]
    assert opt._ns_tiles(big) == 8 * 16 * 16
