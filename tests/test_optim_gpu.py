"""Muon and Dion on CUDA (tcgen05 kernels) vs the float64 oracle."""
import pytest
import torch

from dion_b200 import ops
from dion_b200.optim import Dion, Muon, oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(256, 128), (128, 384), (200, 96)])
def test_muon_cuda_vs_oracle(shape):
    torch.manual_seed(1)
    X = torch.randn(shape, device="cuda")
    G = torch.randn(shape, device="cuda")
    ps = [torch.nn.Parameter(X.clone()) for _ in range(3)]
    opt = Muon(ps, lr=0.02, mu=0.9, weight_decay=0.1, ns_coeffs="keller")
    for p in ps:
        p.grad = G.clone()
    opt.step()
    torch.cuda.synchronize()
    ops.check_status()
    Xr, Mr = oracle.muon_step(X.cpu(), G.cpu(), torch.zeros(shape), 0.02, 0.9, 0.1, False, ops.KELLER_NS_COEFFS)
    for p in ps:
        rel = (p.detach().cpu().double() - Xr).norm() / (Xr - X.cpu().double()).norm()
        assert rel < 0.05, rel


@pytest.mark.parametrize("shape", [(512, 256), (256, 768), (384, 384)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_dion_cuda_vs_oracle(shape, dtype):
    torch.manual_seed(2)
    X = torch.randn(shape, device="cuda")
    G = torch.randn(shape, device="cuda")
    ps = [torch.nn.Parameter(X.clone().to(dtype)) for _ in range(2)]
    opt = Dion(ps, lr=0.02, mu=0.9, weight_decay=0.1, rank_fraction=0.25)
    for p in ps:
        p.grad = G.clone().to(dtype)
    for p in ps:
        opt._get_or_initialize_state(p, opt.param_groups[0])
    Q0 = [opt.state[p]["Q"].detach().clone() for p in ps]
    opt.step()
    torch.cuda.synchronize()
    ops.check_status()
    for p, q0 in zip(ps, Q0):
        Xr, Mr, Qr = oracle.dion_step(X.to(dtype).cpu(), G.to(dtype).cpu(), torch.zeros(shape), q0.cpu(),
                                      0.02, 0.9, 0.1)
        dm = (opt.state[p]["momentum"].cpu().double() - Mr).norm() / Mr.norm()
        assert dm < 2e-2, dm
        if dtype == torch.float32:
            dx = (p.detach().cpu().double() - Xr).norm() / (Xr - X.cpu().double()).norm()
            assert dx < 2e-2, dx
        else:
            # bf16 weights: the step is below bf16 resolution of X, compare at that resolution
            torch.testing.assert_close(p.detach().cpu().double(), Xr, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
def test_effective_rank_kernel_matches_torch():
    from dion_b200 import ops

    torch.manual_seed(0)
    sumsq = torch.rand(12, 96, device="cuda") ** 3
    sumsq[3, 5] = -1e-9  # rounding can leave tiny negatives: clamped
    slots = torch.tensor([0, 3, 7, 11, 5], device="cuda")
    ranks = torch.tensor([96, 40, 1, 64, 17], device="cuda", dtype=torch.int32)
    got = ops.effective_rank(sumsq, slots, ranks)
    ref = ops.effective_rank(sumsq.cpu().double(), slots.cpu(), ranks.cpu())
    torch.testing.assert_close(got.cpu().double(), ref, rtol=1e-4, atol=1e-4)
    assert abs(float(got[2]) - 1.0) < 1e-4  # one active column: effective rank 1


@pytest.mark.gpu
@pytest.mark.parametrize("r", [64, 30])
@pytest.mark.parametrize("qdtype", [torch.float32, torch.bfloat16])
def test_column_norm_kernels(r, qdtype):
    """col_sumsq / col_normalize (vector path when r % 4 == 0, scalar otherwise;
    output into a strided view of a wider buffer) against torch fp32."""
    from dion_b200 import ops

    torch.manual_seed(0)
    R = torch.randn(3, 1000, r, device="cuda")
    s = ops.col_sumsq(R)
    torch.testing.assert_close(s, R.square().sum(dim=1), rtol=1e-5, atol=1e-4)
    wide = torch.zeros(3, 1000, r + 8, device="cuda", dtype=qdtype)
    Q = wide[:, :, :r]
    ops.col_normalize(R, s, 1e-8, Q)
    ref = R / (s.sqrt().unsqueeze(1) + 1e-8)
    tol = 1e-5 if qdtype == torch.float32 else 1e-2
    torch.testing.assert_close(Q.float(), ref, rtol=tol, atol=tol)
    assert float(wide[:, :, r:].abs().max()) == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("n", [4096, 1001, 3])
def test_philox_kernel_matches_cpu_oracle(n):
    from dion_b200 import ops

    for key, stream in ((0, 0), (1234567, 42), ((1 << 64) - 5, (1 << 63) + 7)):
        g = ops.philox_normal((n,), key, stream, 0.5, "cuda")
        c = ops.philox_normal((n,), key, stream, 0.5, "cpu")
        torch.testing.assert_close(g.cpu(), c, rtol=1e-5, atol=1e-5)
        assert torch.equal(g, ops.philox_normal((n,), key, stream, 0.5, "cuda"))
