"""Device-side failure detection without a GPU fault: the peer barrier of the
symmetric-memory collectives waits on a flag that nothing sets (a peer that
never arrives), gives up after a short limit, reports through the status
word, and leaves the context usable."""
import pytest
import torch

from dion_b200 import ops

pytestmark = pytest.mark.gpu

COMM_TIMEOUT = 0x201


def test_barrier_peer_never_arrives_reports_timeout():
    E = ops.ext()
    ptr, _ = E.symm_create(1 << 21)
    old = E.wait_limit_ns()
    try:
        # a 2-rank world whose "peer" flag area is this GPU's own region: slot 0
        # receives both arrivals, slot 1 (the absent peer's) is never written
        flags = torch.tensor([ptr, ptr], dtype=torch.int64, device="cuda")
        E.set_wait_limit_ns(50_000_000)
        E.status_clear()
        E.symm_barrier(flags, ptr, 0, 2)
        torch.cuda.synchronize()
        assert E.status_read() == COMM_TIMEOUT
        with pytest.raises(ops.StatusError):
            ops.check_status()
        E.status_clear()
        # the context is still usable
        x = torch.arange(8, device="cuda", dtype=torch.float32)
        assert float(x.sum()) == 28.0
        # a 1-rank barrier completes without error
        E.symm_barrier(flags[:1].contiguous(), ptr, 0, 1)
        torch.cuda.synchronize()
        assert E.status_read() == 0
    finally:
        E.set_wait_limit_ns(old)
        E.status_clear()
        torch.cuda.synchronize()
        E.symm_free(ptr)
