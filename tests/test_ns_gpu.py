"""Batched Newton-Schulz kernel vs a plain PyTorch fp32 reference."""
import pytest
import torch

from dion_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(4, 256, 768), (3, 768, 256), (2, 512, 512), (1, 1024, 4096), (2, 100, 36)])
@pytest.mark.parametrize("coeffs", ["keller", "dion"])
def test_newton_schulz(shape, coeffs):
    torch.manual_seed(0)
    co = ops.KELLER_NS_COEFFS if coeffs == "keller" else ops.DION_NS_COEFFS
    U = torch.randn(*shape, device="cuda").bfloat16()
    out = ops.newton_schulz(U, co, eps=1e-7)
    ref = ops._ns_reference(U, co, 1e-7)
    torch.cuda.synchronize()
    ops.check_status()
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    # bf16 iterations vs fp32 oracle
    assert rel < 0.05, rel


def test_muon_momentum_and_update():
    torch.manual_seed(0)
    shapes = [(64, 96), (128, 40), (7, 13)]
    M = [torch.randn(s, device="cuda") for s in shapes]
    G = [torch.randn(s, device="cuda").bfloat16() for s in shapes]
    U = [torch.empty(s, device="cuda", dtype=torch.bfloat16) for s in shapes]
    Mc = [m.cpu().clone() for m in M]
    Gc = [g.cpu().clone() for g in G]
    Uc = [u.cpu().clone() for u in U]
    ss, sc = ops.muon_momentum_(M, G, U, 0.9, True, 1e-7)
    ssc, scc = ops.muon_momentum_(Mc, Gc, Uc, 0.9, True, 1e-7)
    for a, b in zip(M, Mc):
        torch.testing.assert_close(a.cpu(), b, rtol=1e-5, atol=1e-5)
    for a, b in zip(U, Uc):
        torch.testing.assert_close(a.cpu().float(), b.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(ss.cpu(), ssc, rtol=1e-4, atol=1e-3)
    X = [torch.randn(s, device="cuda") for s in shapes]
    Xc = [x.cpu().clone() for x in X]
    ops.scaled_update_(X, U, 0.99, [0.1, 0.2, 0.3])
    ops.scaled_update_(Xc, Uc, 0.99, [0.1, 0.2, 0.3])
    for a, b in zip(X, Xc):
        torch.testing.assert_close(a.cpu(), b, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("cautious", [False, True])
def test_adamw_lion(cautious):
    torch.manual_seed(0)
    shapes = [(1000,), (33, 17), (4096, 8)]
    mk = lambda: [torch.randn(s, device="cuda") for s in shapes]
    X, G, M, V = mk(), mk(), mk(), [t.abs() for t in mk()]
    Xc, Gc, Mc, Vc = [[t.cpu().clone() for t in L] for L in (X, G, M, V)]
    ops.adamw_(X, G, M, V, 1e-3, 0.9, 0.95, 0.1, 1e-8, 3, cautious)
    ops.adamw_(Xc, Gc, Mc, Vc, 1e-3, 0.9, 0.95, 0.1, 1e-8, 3, cautious)
    for a, b in zip(X + M + V, Xc + Mc + Vc):
        torch.testing.assert_close(a.cpu(), b, rtol=1e-5, atol=1e-6)
    ops.lion_(X, G, M, 1e-3, 0.9, 0.99, 0.1, cautious)
    ops.lion_(Xc, Gc, Mc, 1e-3, 0.9, 0.99, 0.1, cautious)
    for a, b in zip(X + M, Xc + Mc):
        torch.testing.assert_close(a.cpu(), b, rtol=1e-5, atol=1e-6)
