"""Sequence-parallel tensor parallelism with the TP collectives fused into the
GEMMs over NVLink peer memory.

Layout (Megatron sequence parallelism): between transformer sublayers every
TP rank holds a contiguous shard of the flattened tokens ([N / T, D] of the
batch's N = b * s tokens); norms, residual adds and the embedding run on
that shard. Around each sublayer:

  * column-parallel linears (wq/wk/wv, w1/w3): all-gather of the normalised
    shard, then local GEMMs with the TP-local weight blocks;
  * row-parallel linears (wo, w2): the GEMM of the TP-local input block
    against the TP-local weight block gives a partial [N, D]; its epilogue
    stores the rows of token shard j straight into rank j's receive slot
    (fp32, one slot per source rank), a device barrier orders the stores and
    each rank sums its T slots in a fixed order (reduce-scatter fused into the
    GEMM, no staging copy);
  * the backward mirrors them: the column-parallel input gradient is one
    GEMM over the concatenated output gradients with the same fused
    reduce-scatter epilogue, and the row-parallel output gradient is
    all-gathered before its two GEMMs.

The all-gather pushes each rank's shard into every peer's buffer with plain
16-byte P2P stores; the GEMMs only ever read this GPU's memory. Buffers
alternate between two halves per collective kind, so one barrier per call
orders both the data and the reuse: a rank writing call t's data has passed
call t-1's barrier, which every peer reaches only after consuming call t-2's
data from the same half.

Without peer memory (CPU, gloo, more than one node, or DION_B200_P2P=0) the
same functions run on ``all_gather_into_tensor`` / ``reduce_scatter_tensor``.

Reference counterpart: TP is registered but never enabled in the reference's
configs (ada_dion/integration/config_registry.py:92-103); torchtitan's plan
applies ``SequenceParallel`` + ``ColwiseParallel(input_layouts=Shard(1))`` /
``RowwiseParallel(output_layouts=Shard(1))`` over NCCL.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

from .. import ops

__all__ = ["SPGroup", "sp_column_linears", "sp_row_linear"]


def _mm(a: Tensor, b: Tensor) -> Tensor:
    """``a @ b`` on the package's GEMM for CUDA bf16 operands (torch otherwise)."""
    if a.is_cuda and a.dtype == torch.bfloat16 and ops.has_ext():
        return ops.matmul(a, b)
    return a @ b


class SPGroup:
    """One TP group's sequence-parallel collectives (see the module doc)."""

    def __init__(self, group, device: torch.device):
        from .symm import p2p_enabled

        self.group = group
        self.T = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.device = device
        self.p2p = p2p_enabled(group, device)
        self._heap = None
        self._parity = {"ag": 1, "rs": 1}
        self._ptr_cache: dict = {}
        self.batch_shape: Tuple[int, int] = (0, 0)  # (b, s) of the current step's full token layout

    # ------------------------------------------------------------ token shards
    def shard_rows(self, x: Tensor) -> Tensor:
        """This rank's contiguous block of rows of a [N, ...] tensor."""
        if x.shape[0] % self.T:
            raise ValueError(f"sequence parallelism over {self.T} ranks needs the batch's token count "
                             f"(batch x sequence length = {x.shape[0]}) to be a multiple of {self.T}")
        n = x.shape[0] // self.T
        return x[self.me * n:(self.me + 1) * n]

    # ------------------------------------------------------------ peer memory
    def _layout(self, N: int, D: int):
        ag_half = N * D * 2
        rs_half = N * D * 4
        return ag_half, rs_half, 2 * ag_half + 2 * rs_half

    def _heap_for(self, N: int, D: int):
        from .symm import heap_for

        _, _, need = self._layout(N, D)
        self._heap = heap_for(self.group, need, f"sp:{N}x{D}", self.device)
        return self._heap

    def _flip(self, kind: str) -> int:
        self._parity[kind] = 1 - self._parity[kind]
        return self._parity[kind]

    def all_gather(self, x: Tensor) -> Tensor:
        """[n, D] bf16 shard -> [T * n, D] (rank-major). On peer memory the
        result is a view of this rank's buffer, valid until the next-but-one
        all-gather: consume it right away."""
        n, D = x.shape
        N = n * self.T
        if not self.p2p:
            out = torch.empty((N, D), device=x.device, dtype=x.dtype)
            dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
            return out
        heap = self._heap_for(N, D)
        ag_half, _, _ = self._layout(N, D)
        p = self._flip("ag")
        base = p * ag_half
        key = ("ag", heap.uid, p, n, D)
        ptrs = self._ptr_cache.get(key)
        if ptrs is None:
            ptrs = heap.ptr_tensor([heap.addr(j, base + self.me * n * D * 2) for j in range(self.T)])
            self._ptr_cache[key] = ptrs
            heap.on_close(lambda: self._ptr_cache.pop(key, None))
        heap.push(x.contiguous(), ptrs)
        heap.barrier()
        return heap.view(base, (N, D), x.dtype)

    def gemm_reduce_scatter(self, A: Tensor, B: Tensor) -> Tensor:
        """Row block ``me`` of ``sum over TP ranks of A @ B`` ([N, D] partials
        -> [N / T, D] bf16): the GEMM epilogue stores every row block straight
        into its owner's receive slot."""
        N, D = A.shape[0], B.shape[1]
        n = N // self.T
        if not self.p2p:
            part = (A.float() @ B.float()) if not A.is_cuda else ops.matmul(A, B, out_dtype=torch.float32)
            out = torch.empty((n, D), device=A.device, dtype=torch.float32)
            dist.reduce_scatter_tensor(out, part.float().contiguous(), group=self.group)
            return out.to(A.dtype)
        heap = self._heap_for(N, D)
        ag_half, rs_half, _ = self._layout(N, D)
        p = self._flip("rs")
        base = 2 * ag_half + p * rs_half
        key = ("rs", heap.uid, p, n, D)
        ptrs = self._ptr_cache.get(key)
        if ptrs is None:
            # row block j of my partial -> slot `me` of rank j
            ptrs = heap.ptr_tensor([heap.addr(j, base + self.me * n * D * 4) for j in range(self.T)])
            self._ptr_cache[key] = ptrs
            heap.on_close(lambda: self._ptr_cache.pop(key, None))
        # rotate the row-tile order so ranks start on different destinations
        ops.matmul_to_ptrs(A, B, ptrs, D, torch.float32, rows_per_ptr=n, rot_rows=((self.me + 1) % self.T) * n)
        heap.barrier()
        slots = heap.view(base, (self.T, n, D), torch.float32)
        out = torch.empty((n, D), device=A.device, dtype=torch.float32)
        heap.reduce_slots(slots, out, self.T)
        return out.to(A.dtype)


class _ColumnLinears(torch.autograd.Function):
    """all-gather(x shard) then y_i = x_full @ W_i^T for each TP-local weight."""

    @staticmethod
    def forward(ctx, sp: SPGroup, x: Tensor, *Ws: Tensor):
        x_full = sp.all_gather(x)
        ys = tuple(_mm(x_full, W.t()) for W in Ws)
        ctx.sp = sp
        ctx.save_for_backward(x, *Ws)
        return ys

    @staticmethod
    def backward(ctx, *dys: Tensor):
        sp = ctx.sp
        x, *Ws = ctx.saved_tensors
        dys = [dy.contiguous() for dy in dys]
        x_full = sp.all_gather(x)  # gathered again: the forward's buffer has been reused since
        dWs = [_mm(dy.t(), x_full) for dy in dys]
        dcat = dys[0] if len(dys) == 1 else torch.cat(dys, dim=1)
        Wcat = Ws[0] if len(Ws) == 1 else torch.cat(list(Ws), dim=0)
        dx = sp.gemm_reduce_scatter(dcat, Wcat)
        return (None, dx, *dWs)


class _RowLinear(torch.autograd.Function):
    """y shard = reduce-scatter(x_local @ W^T) with the scatter in the GEMM epilogue."""

    @staticmethod
    def forward(ctx, sp: SPGroup, x: Tensor, W: Tensor):
        x = x.contiguous()
        ctx.sp = sp
        ctx.save_for_backward(x, W)
        return sp.gemm_reduce_scatter(x, W.t())

    @staticmethod
    def backward(ctx, dy: Tensor):
        sp = ctx.sp
        x, W = ctx.saved_tensors
        dy_full = sp.all_gather(dy.contiguous())
        dx = _mm(dy_full, W)
        dW = _mm(dy_full.t(), x)
        return None, dx, dW


def _local(w: Tensor) -> Tensor:
    from torch.distributed.tensor import DTensor

    return w.to_local() if isinstance(w, DTensor) else w


def sp_column_linears(sp: SPGroup, x: Tensor, weights: Sequence[Tensor]) -> List[Tensor]:
    """Column-parallel linears on a sequence shard ``x`` [n, D]: returns the
    [N, out_i / T] outputs for the full token range."""
    return list(_ColumnLinears.apply(sp, x, *[_local(w) for w in weights]))


def sp_row_linear(sp: SPGroup, x: Tensor, weight: Tensor) -> Tensor:
    """Row-parallel linear on the full token range ``x`` [N, in / T]: returns
    this rank's [N / T, out] sequence shard of the summed output."""
    return _RowLinear.apply(sp, x, _local(weight))
