"""Batched Cholesky, triangular inverse and Householder QR kernels vs
float64 PyTorch references."""
import pytest
import torch

from dion_b200 import ops

pytestmark = pytest.mark.gpu


def _spd(b, r, cond=1e3):
    g = torch.Generator(device="cuda").manual_seed(0)
    Q, _ = torch.linalg.qr(torch.randn(b, r, r, device="cuda", dtype=torch.float64, generator=g))
    ev = torch.logspace(0, -torch.log10(torch.tensor(cond)).item(), r, device="cuda", dtype=torch.float64)
    return (Q * ev.unsqueeze(1)) @ Q.mT


@pytest.mark.parametrize("r", [32, 100, 256, 1024])
def test_cholesky_lower(r):
    A = _spd(3, r)
    W = A.float().contiguous()
    info = torch.zeros(3, dtype=torch.int32, device="cuda")
    ops.ext().cholesky_lower(W, info)
    torch.cuda.synchronize()
    L = torch.tril(W).double()
    assert int(info.sum()) == 0
    rel = ((L @ L.mT - A).norm() / A.norm()).item()
    assert rel < 1e-5, rel


def test_cholesky_not_pd_flags():
    A = -torch.eye(64, device="cuda").unsqueeze(0).repeat(2, 1, 1).contiguous()
    info = torch.zeros(2, dtype=torch.int32, device="cuda")
    ops.ext().cholesky_lower(A, info)
    torch.cuda.synchronize()
    assert info.tolist() == [1, 1]
    assert torch.isnan(A).any()


@pytest.mark.parametrize("r", [32, 77, 96, 600, 1024])
@pytest.mark.parametrize("upper", [False, True])
def test_tri_inv(r, upper):
    g = torch.Generator(device="cuda").manual_seed(1)
    L = torch.tril(torch.randn(2, r, r, device="cuda", generator=g)) / r**0.5
    L.diagonal(dim1=1, dim2=2).copy_(1.0 + torch.rand(2, r, device="cuda", generator=g))
    S = (L.mT if upper else L).contiguous()
    Z = torch.empty_like(S)
    ops.ext().tri_inv_lower(S, Z, upper)
    torch.cuda.synchronize()
    eye = torch.eye(r, device="cuda", dtype=torch.float64)
    err = (L.double() @ Z.double() - eye).norm() / r**0.5
    assert err < 1e-4, err
    assert torch.equal(torch.triu(Z, 1), torch.zeros_like(Z))


@pytest.mark.parametrize("mn", [(64, 32), (300, 100), (1280, 1024)])
def test_qr_r(mn):
    m, n = mn
    g = torch.Generator(device="cuda").manual_seed(2)
    A = torch.randn(2, m, n, device="cuda", generator=g)
    W = A.clone()
    R = torch.empty(2, n, n, device="cuda")
    ops.ext().qr_r(W, R)
    torch.cuda.synchronize()
    # R^T R = A^T A and R upper triangular
    G = A.double().mT @ A.double()
    rel = ((R.double().mT @ R.double() - G).norm() / G.norm()).item()
    assert rel < 1e-5, rel
    assert torch.equal(torch.tril(R, -1), torch.zeros_like(R))
    Rref = torch.linalg.qr(A.double(), mode="r")[1]
    torch.testing.assert_close(R.double().abs(), Rref.abs(), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("shape", [(4, 2048, 256), (2, 14336, 1024)])
def test_orthogonalize_kernels(shape):
    from dion_b200.optim.linalg import orthogonalize

    g = torch.Generator(device="cuda").manual_seed(3)
    b, d, r = shape
    # ill-conditioned P, as produced by a power iteration on low-rank momentum
    U, _ = torch.linalg.qr(torch.randn(b, d, r, device="cuda", generator=g))
    s = torch.logspace(0, -4, r, device="cuda")
    V, _ = torch.linalg.qr(torch.randn(b, r, r, device="cuda", generator=g))
    P = (U * s) @ V.mT
    O = orthogonalize(P)
    torch.cuda.synchronize()
    eye = torch.eye(r, device="cuda", dtype=torch.float64)
    orth = (O.double().mT @ O.double() - eye).norm() / r**0.5
    assert orth < 1e-2, orth
    # same column space as P: projecting P onto span(O) recovers P
    proj = O.double() @ (O.double().mT @ P.double())
    assert ((proj - P.double()).norm() / P.double().norm()).item() < 1e-3


# ---------------------------------------------------------------- blocked kernels (tcgen05 3xTF32 trailing updates)
@pytest.mark.parametrize("mn", [(64, 32), (300, 100), (1280, 1024), (2600, 2048), (3000, 200)])
def test_qr_r_blocked(mn):
    """R^T R = A^T A to fp32 accuracy; (2600, 2048) and (3000, 200) split the
    panel rows over a thread-block cluster; n % 32 != 0 exercises the last
    narrow panel."""
    m, n = mn
    g = torch.Generator(device="cuda").manual_seed(2)
    A = torch.randn(3, m, n, device="cuda", generator=g)
    W = A.clone()
    R = torch.empty(3, n, n, device="cuda")
    ops.ext().qr_r_blocked(W, R)
    torch.cuda.synchronize()
    G = A.double().mT @ A.double()
    rel = ((R.double().mT @ R.double() - G).norm() / G.norm()).item()
    assert rel < 2e-6, rel
    assert torch.equal(torch.tril(R, -1), torch.zeros_like(R))
    Rref = torch.linalg.qr(A.double(), mode="r")[1]
    torch.testing.assert_close(R.double().abs(), Rref.abs(), rtol=2e-3, atol=2e-3)


def test_qr_r_blocked_ill_conditioned():
    """Graded columns (condition 1e6): the R factor must still satisfy
    A = Q R with orthonormal Q = A R^-1 to fp32-level backward error."""
    g = torch.Generator(device="cuda").manual_seed(5)
    b, m, n = 2, 1280, 512
    U, _ = torch.linalg.qr(torch.randn(b, m, n, device="cuda", dtype=torch.float64, generator=g))
    V, _ = torch.linalg.qr(torch.randn(b, n, n, device="cuda", dtype=torch.float64, generator=g))
    A = ((U * torch.logspace(0, -6, n, device="cuda", dtype=torch.float64)) @ V.mT).float()
    W = A.clone()
    R = torch.empty(b, n, n, device="cuda")
    ops.ext().qr_r_blocked(W, R)
    torch.cuda.synchronize()
    G = A.double().mT @ A.double()
    rel = ((R.double().mT @ R.double() - G).norm() / G.norm()).item()
    assert rel < 2e-6, rel


@pytest.mark.parametrize("r", [32, 100, 256, 1024, 2048])
def test_cholesky_blocked(r):
    A = _spd(3, r)
    W = A.float().contiguous()
    info = torch.full((3,), 7, dtype=torch.int32, device="cuda")
    ops.ext().cholesky_blocked(W, info)
    torch.cuda.synchronize()
    L = torch.tril(W).double()
    assert info.tolist() == [0, 0, 0]
    rel = ((L @ L.mT - A).norm() / A.norm()).item()
    assert rel < 2e-6, rel


def test_cholesky_blocked_not_pd_flags():
    A = torch.eye(96, device="cuda").unsqueeze(0).repeat(2, 1, 1).contiguous()
    A[1, 40, 40] = -1.0
    info = torch.zeros(2, dtype=torch.int32, device="cuda")
    ops.ext().cholesky_blocked(A, info)
    torch.cuda.synchronize()
    assert info.tolist() == [0, 1]
    assert torch.isnan(A[1]).any() and not torch.isnan(torch.tril(A[0])).any()


def test_orthogonalize_square_on_kernels():
    """d == r (the reference's QR branch) runs the randomised path on the
    kernels: orthonormal columns spanning the same space as P."""
    from dion_b200.optim.linalg import orthogonalize

    g = torch.Generator(device="cuda").manual_seed(6)
    P = torch.randn(3, 512, 512, device="cuda", generator=g)
    O = orthogonalize(P)
    torch.cuda.synchronize()
    eye = torch.eye(512, device="cuda", dtype=torch.float64)
    assert ((O.double().mT @ O.double() - eye).norm() / 512 ** 0.5).item() < 1e-2
    Qref, _ = torch.linalg.qr(P.double())
    # same factor up to column signs
    torch.testing.assert_close(O.double().abs(), Qref.abs(), rtol=0, atol=2e-2)
