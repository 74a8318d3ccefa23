"""Fused model kernels (RMSNorm, RoPE, SwiGLU, cross-entropy) vs PyTorch fp32."""
import pytest
import torch
import torch.nn.functional as F

from dion_b200.models import layers as L
from dion_b200.ops import fused

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,dim", [(37, 512), (3001, 2048), (700, 4096)])
def test_rmsnorm_fwd_bwd(rows, dim):
    """dim >= 1024 takes the row-per-CTA backward kernel (several rows per CTA)."""
    torch.manual_seed(0)
    x = torch.randn(rows, dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(dim, device="cuda", dtype=torch.float32, requires_grad=True)
    y = fused.rms_norm(x, w, 1e-5)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    yr = F.rms_norm(xr, (dim,), wr, 1e-5)
    yr.backward(g.float())
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad, wr.grad, rtol=1e-2, atol=1e-1 * (rows / 37) ** 0.5)


@pytest.mark.parametrize("b,s,hq,hk,d", [(2, 64, 8, 2, 64), (3, 257, 32, 8, 128)])
def test_rope_roundtrip_and_ref(b, s, hq, hk, d):
    torch.manual_seed(0)
    q = torch.randn(b, s, hq, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(b, s, hk, d, device="cuda", dtype=torch.bfloat16)
    tab = L.rope_table(d, 2 * s, 10000.0).cuda()
    qo, ko = fused.rope(q, k, tab)
    torch.testing.assert_close(qo.float(), L._rope_ref(q, tab).float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(ko.float(), L._rope_ref(k, tab).float(), rtol=2e-2, atol=2e-2)
    qr = q.clone().requires_grad_()
    kr = k.clone().requires_grad_()
    a, b = fused.rope(qr, kr, tab)
    (a.float().sum() + 2 * b.float().sum()).backward()
    q2 = q.float().requires_grad_()
    k2 = k.float().requires_grad_()
    (L._rope_ref(q2, tab).sum() + 2 * L._rope_ref(k2, tab).sum()).backward()
    torch.testing.assert_close(qr.grad.float(), q2.grad, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(kr.grad.float(), k2.grad, rtol=2e-2, atol=2e-2)


def test_swiglu():
    torch.manual_seed(0)
    a = torch.randn(64, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    b = torch.randn(64, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = fused.swiglu(a, b)
    g = torch.randn_like(o)
    o.backward(g)
    af, bf = a.detach().float().requires_grad_(), b.detach().float().requires_grad_()
    of = F.silu(af) * bf
    of.backward(g.float())
    torch.testing.assert_close(o.float(), of, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(a.grad.float(), af.grad, rtol=2e-2, atol=3e-2)
    torch.testing.assert_close(b.grad.float(), bf.grad, rtol=2e-2, atol=3e-2)


def test_linear_cross_entropy():
    torch.manual_seed(0)
    T, d, V = 300, 256, 4096
    h = (torch.randn(T, d, device="cuda") * 0.5).bfloat16().requires_grad_()
    W = (torch.randn(V, d, device="cuda") * 0.05).bfloat16().requires_grad_()
    lab = torch.randint(0, V, (T,), device="cuda")
    loss = L.linear_cross_entropy(h, W, lab, chunk=128)
    loss.backward()
    hf, Wf = h.detach().float().requires_grad_(), W.detach().float().requires_grad_()
    lf = F.cross_entropy(hf @ Wf.t(), lab)
    lf.backward()
    assert abs(loss.item() - lf.item()) < 1e-2
    torch.testing.assert_close(h.grad.float(), hf.grad, rtol=5e-2, atol=5e-3)
    torch.testing.assert_close(W.grad.float(), Wf.grad, rtol=5e-2, atol=5e-3)
    # evaluation (no autograd): the same chunked loss without the gradient products
    W.grad = None
    with torch.no_grad():
        ev = L.linear_cross_entropy(h, W, lab, chunk=128)
    assert W.grad is None and abs(ev.item() - lf.item()) < 1e-2 and abs(ev.item() - loss.item()) < 1e-5


@pytest.mark.parametrize("rows,dim", [(513, 2048), (64, 1024)])
def test_add_rmsnorm_fused(rows, dim):
    """(x + a, rms_norm(x + a) * w) and its backward (the residual gradient added
    to the norm's input gradient) against PyTorch fp32."""
    torch.manual_seed(1)
    x = torch.randn(rows, dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    a = torch.randn(rows, dim, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(dim, device="cuda", dtype=torch.float32, requires_grad=True)
    assert fused.add_rms_enabled(x)
    h, y = fused.add_rms_norm(x, a, w, 1e-5)
    gh, gy = torch.randn_like(h), torch.randn_like(y)
    torch.autograd.backward([h, y], [gh, gy])
    xr = x.detach().float().requires_grad_()
    ar = a.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    hr = (xr + ar).to(torch.bfloat16).float()  # the unfused add rounds to bf16
    yr = F.rms_norm(hr, (dim,), wr, 1e-5)
    torch.autograd.backward([hr, yr], [gh.float(), gy.float()])
    torch.testing.assert_close(h.float(), hr, rtol=0, atol=0)
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(a.grad.float(), ar.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad, wr.grad, rtol=1e-2, atol=1e-1 * (rows / 37) ** 0.5)
