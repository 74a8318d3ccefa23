"""The sequence-parallel collectives' data movement on ONE GPU, with T
virtual ranks whose "peer" buffers are slices of local tensors: the
all-gather pushes, the reduce-scatter fused into the GEMM epilogue (row
blocks to each owner's slot, with the per-rank tile rotation) and the
fixed-order slot sum. The kernels and pointer tables are exactly those of
parallel/sp.py; only the cross-GPU barrier is absent (one stream orders
everything here), so the addressing is checked where no second GPU exists.
The multi-GPU runs are tests/test_parallel_gpu.py."""
import pytest
import torch

from dion_b200 import ops

pytestmark = pytest.mark.gpu


def _ptrs(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


@pytest.mark.parametrize("T", [2, 4])
def test_emulated_gemm_reduce_scatter(T):
    torch.manual_seed(0)
    N, K, D = 1024, 320, 512
    n = N // T
    A = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) for _ in range(T)]  # rank r's input block
    B = [torch.randn(K, D, device="cuda", dtype=torch.bfloat16) for _ in range(T)]  # rank r's weight block
    slots = torch.zeros(T, T, n, D, device="cuda")  # slots[owner, source]
    for r in range(T):  # rank r's GEMM: row block j -> slot r of rank j
        ops.matmul_to_ptrs(A[r], B[r], _ptrs([slots[j, r] for j in range(T)]), D, torch.float32,
                           rows_per_ptr=n, rot_rows=((r + 1) % T) * n)
    full = sum(a.float() @ b.float() for a, b in zip(A, B))
    for j in range(T):
        out = torch.empty(n, D, device="cuda")
        ops.ext().symm_reduce_slots(slots[j].contiguous(), out, T)
        ref = full[j * n:(j + 1) * n]
        assert ((out - ref).norm() / ref.norm()).item() < 1e-2


@pytest.mark.parametrize("T", [2, 4])
def test_emulated_all_gather_push(T):
    torch.manual_seed(1)
    n, D = 96, 256
    shards = [torch.randn(n, D, device="cuda", dtype=torch.bfloat16) for _ in range(T)]
    bufs = torch.zeros(T, T * n, D, device="cuda", dtype=torch.bfloat16)  # every rank's gather buffer
    for r in range(T):  # rank r pushes its shard into rows [r*n, (r+1)*n) of every buffer
        ops.ext().symm_push(shards[r], _ptrs([bufs[j, r * n] for j in range(T)]))
    ref = torch.cat(shards)
    for j in range(T):
        assert torch.equal(bufs[j], ref)
