"""AdaDion, AdaDionV2 and the research variants (SDion, GSDion, AGDion,
QCDion) on CUDA: invariants, convergence, one step against the same
optimizer on CPU from identical state, and the kernels they use for Q
refills (Philox normals + column sum-of-squares + column normalise)."""
import copy

import pytest
import torch
import torch.nn as nn

from dion_b200 import ops
from dion_b200.optim import AGDion, AdaDion, AdaDionV2, GSDion, QCDion, SDion

pytestmark = pytest.mark.gpu

ADAPTIVE = [
    (AdaDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32, warmup_rank=16)),
    (SDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32)),
    (GSDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32, warmup_rank=16)),
    (AGDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32)),
    (QCDion, dict(lr=0.02, init_rank=8, rank_min=4, rank_max=32)),
    (AdaDionV2, dict(lr=0.02, adaptive_rank=True, init_rank_fraction=0.25, rank_min=4)),
]
# fixed rank: no refills, so the CPU and CUDA runs draw no random columns
FIXED = [
    (AdaDion, dict(lr=0.02, init_rank=8, rank_min=8, rank_max=8, warmup_rank=8)),
    (SDion, dict(lr=0.02, init_rank=8, rank_min=8, rank_max=8)),
    (GSDion, dict(lr=0.02, init_rank=8, rank_min=8, rank_max=8, warmup_rank=8)),
    (AGDion, dict(lr=0.02, init_rank=8, rank_min=8, rank_max=8)),
    (QCDion, dict(lr=0.02, init_rank=8, rank_min=8, rank_max=8)),
    (AdaDionV2, dict(lr=0.02, adaptive_rank=False, init_rank_fraction=0.25)),
]


@pytest.mark.parametrize("cls,kw", ADAPTIVE, ids=[c.__name__ for c, _ in ADAPTIVE])
@pytest.mark.parametrize("shape", [(256, 128), (128, 384)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cuda_steps_finite_and_change(cls, kw, shape, dtype):
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(shape, device="cuda", dtype=dtype))
    before = p.detach().clone()
    opt = cls([p], **kw)
    for _ in range(4):
        p.grad = torch.randn_like(p) * 0.1
        opt.step()
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.isfinite(p.float()).all()
    assert not torch.equal(p.detach(), before)


@pytest.mark.parametrize("cls,kw", ADAPTIVE, ids=[c.__name__ for c, _ in ADAPTIVE])
def test_cuda_quadratic_loss_decreases(cls, kw):
    torch.manual_seed(42)
    p = nn.Parameter(torch.randn(128, 256, device="cuda"))
    opt = cls([p], **kw)
    losses = []
    for _ in range(60):
        opt.zero_grad()
        loss = (p**2).sum()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert all(map(lambda v: v == v, losses)) and losses[-1] < losses[0]


@pytest.mark.parametrize("cls,kw", FIXED, ids=[c.__name__ for c, _ in FIXED])
@pytest.mark.parametrize("shape", [(256, 128), (128, 384)])
def test_cuda_step_matches_cpu_from_same_state(cls, kw, shape):
    """Two CPU steps build the state; a CPU and a CUDA optimizer loaded with
    it take the same third step. The update (tf32 tensor-core products on
    CUDA, fp32 on CPU) must agree to a few percent of its norm."""
    torch.manual_seed(0)
    pa = nn.Parameter(torch.randn(shape))
    A = cls([pa], **kw)
    for _ in range(2):
        pa.grad = torch.randn(shape) * 0.1
        A.step()
    pb = nn.Parameter(pa.detach().clone().cuda())
    B = cls([pb], **kw)
    B.load_state_dict(copy.deepcopy(A.state_dict()))
    x0 = pa.detach().clone()
    g = torch.randn(shape) * 0.1
    pa.grad, pb.grad = g.clone(), g.cuda()
    A.step()
    B.step()
    torch.cuda.synchronize()
    da, db = pa.detach() - x0, pb.detach().cpu() - x0
    assert da.norm() > 0
    assert float((da - db).norm() / da.norm()) < 5e-2


def test_random_unit_columns_kernel_matches_oracle():
    """Philox normals (kernel vs the CPU integer-arithmetic oracle) then
    column normalise, written into a column slice of a wider buffer."""
    Q = torch.zeros(300, 40, device="cuda")
    ops.random_unit_columns_(Q[:, 8:20], key=1234, stream=77)
    z = ops.philox_normal((300, 12), 1234, 77, 1.0, "cpu").double()
    ref = z / z.norm(dim=0, keepdim=True)
    got = Q[:, 8:20].double().cpu()
    assert torch.allclose(got, ref, atol=1e-5, rtol=1e-4)
    assert Q[:, :8].abs().sum() == 0 and Q[:, 20:].abs().sum() == 0
    Qb = torch.zeros(64, 24, device="cuda", dtype=torch.bfloat16)
    ops.random_unit_columns_(Qb[:, 4:12])
    n = Qb[:, 4:12].float().norm(dim=0)
    assert torch.allclose(n, torch.ones_like(n), atol=1e-2)


def test_keyed_unit_columns_are_a_function_of_their_key():
    """Keyed refills (used so resumed runs and every rank draw the same
    columns): same key -> same columns, another key -> other columns, and
    the kernel result equals the Philox oracle for that key's stream."""
    Q1 = torch.zeros(200, 16, device="cuda")
    Q2 = torch.zeros(200, 16, device="cuda")
    ops.keyed_unit_columns_(Q1[:, 2:10], 7, 200, 16, 5, 2, 10)
    ops.keyed_unit_columns_(Q2[:, 2:10], 7, 200, 16, 5, 2, 10)
    assert torch.equal(Q1, Q2)
    ops.keyed_unit_columns_(Q2[:, 2:10], 7, 200, 16, 6, 2, 10)
    assert not torch.equal(Q1, Q2)
    z = ops.philox_normal((200, 8), torch.initial_seed(), ops.keyed_stream(7, 200, 16, 5, 2, 10), 1.0, "cpu")
    ref = (z / z.norm(dim=0, keepdim=True)).double()
    assert torch.allclose(Q1[:, 2:10].double().cpu(), ref, atol=1e-5, rtol=1e-4)


LOWRANK_ADAPTIVE = [(c, kw) for c, kw in ADAPTIVE if c is not AdaDionV2]


@pytest.mark.parametrize("cls,kw", LOWRANK_ADAPTIVE, ids=[c.__name__ for c, _ in LOWRANK_ADAPTIVE])
def test_cuda_resume_matches_uninterrupted(cls, kw):
    """Adaptive-rank runs refill Q columns; with keyed refills a run resumed
    from a state dict reproduces the uninterrupted run. (AdaDionV2 is left
    out: its randomised orthogonaliser draws a fresh sketch per call, which
    changes the result only by rounding and column signs.)"""
    torch.manual_seed(1)
    x0 = torch.randn(256, 128, device="cuda")

    def grads(i):
        return torch.randn(256, 128, device="cuda", generator=torch.Generator("cuda").manual_seed(100 + i)) * 0.1

    ref = nn.Parameter(x0.clone())
    R = cls([ref], **kw)
    for i in range(6):
        ref.grad = grads(i)
        R.step()
    a = nn.Parameter(x0.clone())
    A = cls([a], **kw)
    for i in range(3):
        a.grad = grads(i)
        A.step()
    b = nn.Parameter(a.detach().clone())
    B = cls([b], **kw)
    B.load_state_dict(copy.deepcopy(A.state_dict()))
    for i in range(3, 6):
        b.grad = grads(i)
        B.step()
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.allclose(b.detach(), ref.detach(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_col_normalize_2d_matches_fp32(dtype):
    torch.manual_seed(3)
    V = torch.randn(513, 37, device="cuda").to(dtype)
    got = ops.col_normalize_2d(V).float()
    Vf = V.float()
    ref = Vf / Vf.norm(dim=0, keepdim=True)
    assert torch.allclose(got, ref, atol=1e-2 if dtype == torch.bfloat16 else 1e-5)
    sq = Vf.square().sum(dim=0) * 4.0
    half = ops.col_normalize_2d(V, sumsq=sq).float()
    assert torch.allclose(half, ref / 2, atol=1e-2 if dtype == torch.bfloat16 else 1e-5)
