"""Fused model kernels (RMSNorm, RoPE, SwiGLU, cross-entropy) vs PyTorch fp32."""
import pytest
import torch
import torch.nn.functional as F

from dion_b200.models import layers as L
from dion_b200.ops import fused

pytestmark = pytest.mark.gpu


def test_rmsnorm_fwd_bwd():
    torch.manual_seed(0)
    x = torch.randn(37, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(512, device="cuda", dtype=torch.float32, requires_grad=True)
    y = fused.rms_norm(x, w, 1e-5)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    yr = F.rms_norm(xr, (512,), wr, 1e-5)
    yr.backward(g.float())
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad, wr.grad, rtol=1e-2, atol=1e-1)


def test_rope_roundtrip_and_ref():
    torch.manual_seed(0)
    q = torch.randn(2, 64, 8, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(2, 64, 2, 64, device="cuda", dtype=torch.bfloat16)
    tab = L.rope_table(64, 128, 10000.0).cuda()
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
