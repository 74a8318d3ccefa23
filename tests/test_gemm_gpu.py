"""tcgen05 GEMM kernel vs a plain PyTorch fp32 reference."""
import pytest
import torch

from dion_b200 import ops

pytestmark = pytest.mark.gpu


def _ref(A, B, C=None, alpha=1.0, beta=0.0):
    r = alpha * (A.float() @ B.float())
    if C is not None:
        r = r + beta * C.float()
    return r


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.fixture(autouse=True, params=[0, 1], ids=["cta1", "cta_pair"])
def gemm_kernel_mode(request):
    """Every GEMM test runs with the single-CTA kernels and with the CTA-pair
    (cta_group::2) kernels."""
    E = ops.ext()
    old = E.gemm_pair_mode()
    E.set_gemm_pair_mode(request.param)
    yield request.param
    E.set_gemm_pair_mode(old)


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", [(256, 512, 384), (200, 296, 72), (128, 128, 64), (3, 520, 1032, 264)])
def test_gemm_layouts(a_t, b_t, shape):
    torch.manual_seed(0)
    if len(shape) == 3:
        batch, (M, N, K) = 1, shape
    else:
        batch, M, N, K = shape
    dev = "cuda"
    A = torch.randn(batch, K, M, device=dev).bfloat16().transpose(1, 2) if a_t else torch.randn(batch, M, K, device=dev).bfloat16()
    B = torch.randn(batch, N, K, device=dev).bfloat16().transpose(1, 2) if b_t else torch.randn(batch, K, N, device=dev).bfloat16()
    out = ops.matmul(A, B, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_status()
    assert _rel(out, _ref(A, B)) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gemm_epilogue_beta(dtype):
    torch.manual_seed(1)
    A = torch.randn(2, 384, 256, device="cuda").bfloat16()
    B = torch.randn(2, 256, 640, device="cuda").bfloat16()
    C = torch.randn(2, 384, 640, device="cuda").to(dtype)
    out = ops.matmul(A, B, C=C, alpha=0.5, beta=-1.5, out_dtype=dtype)
    torch.cuda.synchronize()
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel(out, _ref(A, B, C, 0.5, -1.5)) < tol


@pytest.mark.parametrize("n", [128, 384, 520, 1024])
def test_gemm_symmetric(n):
    torch.manual_seed(2)
    X = torch.randn(2, n, 328, device="cuda").bfloat16()
    out = torch.full((2, n, n), float("nan"), device="cuda", dtype=torch.float32)
    ops.matmul(X, X.transpose(1, 2), out, symmetric=True)
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    assert _rel(out, _ref(X, X.transpose(1, 2))) < 1e-5


def test_gemm_large_bf16():
    torch.manual_seed(3)
    A = torch.randn(2048, 4096, device="cuda").bfloat16()
    B = torch.randn(4096, 3072, device="cuda").bfloat16()
    out = ops.matmul(A, B)
    torch.cuda.synchronize()
    ops.check_status()
    assert _rel(out, _ref(A, B)) < 1e-2


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", [(256, 512, 384), (200, 296, 72), (2, 1000, 1024, 520)])
def test_gemm_tf32_layouts(a_t, b_t, shape):
    torch.manual_seed(0)
    if len(shape) == 3:
        batch, (M, N, K) = 1, shape
    else:
        batch, M, N, K = shape
    A = torch.randn(batch, K, M, device="cuda").transpose(1, 2) if a_t else torch.randn(batch, M, K, device="cuda")
    B = torch.randn(batch, N, K, device="cuda").transpose(1, 2) if b_t else torch.randn(batch, K, N, device="cuda")
    out = ops.matmul(A, B)
    torch.cuda.synchronize()
    ref = A.double() @ B.double()
    # tf32 operands: ~1e-3 relative
    assert _rel(out.double(), ref) < 2e-3


def test_gemm_ptr_array_param_update():
    """Per-batch output pointers + in-place param update D = g*D + d*(A@B)."""
    from dion_b200.ops import _ext

    torch.manual_seed(4)
    A = torch.randn(3, 256, 64, device="cuda")
    B = torch.randn(3, 64, 320, device="cuda")
    Xs = [torch.randn(256, 320, device="cuda") for _ in range(3)]
    ref = [0.9 * x - 0.1 * (a @ b) for x, a, b in zip(Xs, A.unbind(0), B.unbind(0))]
    ops.matmul_update_(Xs, A, B, gamma=0.9, delta=-0.1)
    torch.cuda.synchronize()
    for x, r in zip(Xs, ref):
        assert _rel(x, r) < 2e-3


@pytest.mark.parametrize("rot_b,rot_rows", [(0, 0), (3, 0), (0, 512), (2, 384)])
def test_matmul_to_ptrs_rotation_and_row_split(rot_b, rot_rows):
    """Pointer-array outputs with the per-rank tile-order rotation: batch and
    row-tile rotations only change the order tiles are produced in, and
    row-split destinations receive exactly their rows (here the destinations
    are slices of one local buffer)."""
    torch.manual_seed(0)
    b, M, K, N, rows_per = 5, 1024, 256, 384, 256
    A = torch.randn(b, M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(b, K, N, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(b, M, N, device="cuda", dtype=torch.float32)
    splits = M // rows_per
    ptrs = torch.tensor([out[i, j * rows_per].data_ptr() for i in range(b) for j in range(splits)],
                        dtype=torch.int64, device="cuda")
    ops.matmul_to_ptrs(A, B, ptrs, N, torch.float32, rows_per_ptr=rows_per, rot_b=rot_b, rot_rows=rot_rows)
    torch.testing.assert_close(out, _ref(A, B), rtol=2e-2, atol=2e-1)
    # replicated destinations: every batch written to two buffers
    out2 = torch.zeros(2, b, M, N, device="cuda", dtype=torch.float32)
    ptrs2 = torch.tensor([out2[r, i].data_ptr() for i in range(b) for r in range(2)], dtype=torch.int64,
                         device="cuda")
    ops.matmul_to_ptrs(A, B, ptrs2, N, torch.float32, nrep=2, rot_b=rot_b, rot_rows=rot_rows)
    torch.testing.assert_close(out2[0], out, rtol=0, atol=0)
    torch.testing.assert_close(out2[1], out, rtol=0, atol=0)


@pytest.mark.parametrize("shape", [(256, 4096, 256), (64, 1000, 96), (3, 512, 300, 64)])
def test_matmul_precise_is_fp32_accurate(shape):
    """3xTF32 on the tensor cores in K chunks: relative error near fp32
    SGEMM's (plain tf32 is ~1e-3)."""
    g = torch.Generator(device="cuda").manual_seed(4)
    *b, m, k, n = shape
    A = torch.randn(*b, m, k, device="cuda", generator=g)
    B = torch.randn(*b, k, n, device="cuda", generator=g)
    ref = A.double() @ B.double()
    out = ops.matmul_precise(A, B)
    rel = ((out.double() - ref).norm() / ref.norm()).item()
    assert rel < 5e-6, rel
    plain = ops.matmul(A, B)
    assert ((plain.double() - ref).norm() / ref.norm()).item() > 10 * rel
