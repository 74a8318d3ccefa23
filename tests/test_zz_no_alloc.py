"""The allocation-free C entry point ``bdion_batched_sumsq_noalloc``.

Some callers of this library cannot allocate device memory when they need a
result: a host runtime that reserved its whole device-memory budget at
start-up, code running inside an allocator or out-of-memory callback, or a
plain C caller without PyTorch's allocator. The entry point serves them with
scratch memory fixed inside the library. This test calls it through its
exported C symbol (ctypes) and checks it, on two calls in a row, against the
extension's existing ``multi_sumsq`` op and against a plain PyTorch fp32
reference (``x.float().square().sum()``). It lives in its own file, collected
last, and runs the same alone or after the rest of the suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, TOO_LARGE = 0, -2


def _entry():
    import dion_b200._C as C

    fn = ctypes.CDLL(C.__file__).bdion_batched_sumsq_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_void_p]
    return fn


def _call(fn, x2d, dtype):
    """Run the entry point on the rows of a 2-D view (row stride may exceed the row length)."""
    out = torch.full((x2d.size(0),), -1.0, device="cuda")
    rc = fn(x2d.data_ptr(), 0 if dtype == torch.float32 else 1, x2d.size(0), x2d.size(1), x2d.stride(0),
            out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return rc, out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_sumsq_matches_existing_op(dtype):
    from dion_b200 import ops

    fn = _entry()
    torch.manual_seed(0)
    for call in range(2):  # two calls in a row share the scratch array
        x = torch.randn(50, 300, 70 + 8 * call, device="cuda").to(dtype)  # > 48 tensors: two launch groups
        ref = ops.multi_sumsq(list(x.unbind(0)))
        torch_ref = x.float().square().sum(dim=(1, 2))
        rc, out = _call(fn, x.view(x.size(0), -1), dtype)
        assert rc == OK
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(out, torch_ref, rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("row_len", [312, 301])  # 16-byte aligned rows (vector loads) / odd stride (scalar loads)
def test_noalloc_sumsq_strided_rows(dtype, row_len):
    """Tensors taken as slices of a larger buffer: stride > numel, and with an
    odd stride the kernel takes its scalar-load path."""
    fn = _entry()
    torch.manual_seed(1)
    for call in range(2):
        buf = torch.randn(100 + call, row_len, device="cuda").to(dtype)
        x = buf[:, :300]  # 100+ tensors of 300 elements, stride row_len
        rc, out = _call(fn, x, dtype)
        assert rc == OK
        torch.cuda.synchronize()
        torch.testing.assert_close(out, x.float().square().sum(dim=1), rtol=1e-5, atol=1e-3)


def test_noalloc_rejects_sizes_beyond_scratch():
    fn = _entry()
    x = torch.zeros(16, device="cuda")
    out = torch.zeros(1, device="cuda")
    # 2^31 elements per tensor need 131072 partials > 65536: refused before any launch
    rc = fn(x.data_ptr(), 0, 1, 1 << 31, 1 << 31, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
