"""Dion2 selection / update kernels against plain PyTorch (fp32)."""
import pytest
import torch

from dion_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,k", [((256, 96), 64), ((1000, 40), 1), ((3000, 64), 750), ((128, 32), 128)])
def test_select_gather_update(dtype, shape, k):
    g = torch.Generator(device="cuda").manual_seed(0)
    rows, cols = shape
    M = [torch.randn(rows, cols, device="cuda", generator=g).to(dtype) for _ in range(5)]
    X = [torch.randn(rows, cols, device="cuda", generator=g).to(dtype) for _ in range(5)]
    M0 = [m.clone() for m in M]
    X0 = [x.clone() for x in X]
    idx, pos = ops.dion2_select_rows(M, k)
    for b in range(5):
        score = M0[b].float().abs().sum(dim=1)
        ref = score.topk(k).indices.sort().values
        assert torch.equal(idx[b], ref), b
        p = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        p[ref] = torch.arange(k, dtype=torch.int32, device="cuda")
        assert torch.equal(pos[b], p)
    sel = ops.dion2_gather_decay_(M, idx, 0.5)
    for b in range(5):
        torch.testing.assert_close(sel[b].float(), M0[b][idx[b]].bfloat16().float(), rtol=0, atol=0)
        exp = M0[b].float().clone()
        exp[idx[b]] *= 0.5
        torch.testing.assert_close(M[b].float(), exp.to(dtype).float(), rtol=0, atol=0)
    U = torch.randn(5, k, cols, device="cuda", generator=g).bfloat16()
    ops.dion2_update_(X, pos, U, 0.9, 0.1)
    for b in range(5):
        exp = 0.9 * X0[b].float()
        exp[idx[b]] -= 0.1 * U[b].float()
        tol = 1e-6 if dtype == torch.float32 else 1e-2
        torch.testing.assert_close(X[b].float(), exp, rtol=tol, atol=tol)


def test_topk_ties_take_lowest_rows():
    s = torch.zeros(2, 4096, device="cuda")
    s[0, 100:200] = 1.0  # 100 equal scores, 40 wanted: rows 100..139
    s[1] = torch.arange(4096, device="cuda").float() % 7
    idx = torch.empty(2, 40, dtype=torch.int64, device="cuda")
    pos = torch.empty(2, 4096, dtype=torch.int32, device="cuda")
    ops.ext().dion2_topk_rows(s, 40, idx, pos)
    assert idx[0].tolist() == list(range(100, 140))
    # row 2: 585 rows score 6; the 40 lowest of them
    assert idx[1].tolist() == [i for i in range(4096) if i % 7 == 6][:40]
    assert int((pos[0] >= 0).sum()) == 40


def test_dion2_optimizer_kernels_match_cpu():
    """A Dion2 step on the GPU (kernels) equals the CPU definition."""
    from dion_b200.optim import Dion2

    torch.manual_seed(0)
    ws = [torch.randn(192, 64) for _ in range(3)]
    gs = [torch.randn(192, 64) for _ in range(3)]
    res = {}
    for dev in ("cpu", "cuda"):
        ps = [torch.nn.Parameter(w.clone().to(dev)) for w in ws]
        opt = Dion2(ps, lr=0.02, fraction=0.25, weight_decay=0.1)
        for _ in range(3):
            for p, gr in zip(ps, gs):
                p.grad = gr.to(dev).clone()
            opt.step()
        res[dev] = [p.detach().cpu() for p in ps]
    for a, b in zip(res["cpu"], res["cuda"]):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-3)
