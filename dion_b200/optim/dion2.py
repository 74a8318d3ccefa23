"""Dion2: Newton-Schulz on an alpha-fraction of momentum rows.

Per matrix and step (the method named in the reference paper,
paper/main.tex:70, and exercised by ada_dion/tests/test_dion2.py; the
dion package build installed next to the reference does not ship it, so
the rule below is this package's statement of it):

    M += G
    S = the ceil(fraction * rows) rows of M with the largest L1 norm
        (selection_method="top_l1") or a uniform random subset ("random")
    U = NewtonSchulz(M[S])                   (k x cols, bf16 tensor cores)
    X = (1 - lr*wd) X                        (weight decay on every row)
    X[S] -= lr * sqrt(fan_out/fan_in) * U    (Muon's spectral-norm scaling)
    M[S] *= ef_decay                         (selective decay: only used rows)

Unselected rows keep accumulating, so every row is eventually applied (error
feedback). Sharded layouts:
  * FSDP (rows sharded over W ranks): each rank picks its top rows locally
    (ceil(fraction * rows/W) per shard, balanced traffic) and one all-to-all
    per shape group carries the selected rows to the matrix owner and back,
    i.e. ``fraction`` of Muon's all-to-all volume;
  * DDP: replicas orthogonalise their own matrices and all-gather the rows.
"""
from __future__ import annotations

import math
from typing import Any, Dict, List, Optional, Tuple, Union

import torch
import torch.distributed as dist
from torch import Tensor
from torch.distributed import ProcessGroup
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor import DTensor
from torch.optim.optimizer import Optimizer, ParamsT

from .. import ops
from ..utils.trace import phase
from ._utils import group_by_signature, scalar_update, to_local
from .muon import _ADJUST, _resolve_coeffs

__all__ = ["Dion2"]


class Dion2(Optimizer):
    def __init__(
        self,
        params: ParamsT,
        distributed_mesh: Optional[Union[DeviceMesh, ProcessGroup]] = None,
        lr: float = 0.01,
        fraction: float = 0.25,
        ef_decay: float = 0.95,
        betas: Tuple[float, float] = (0.9, 0.95),
        weight_decay: float = 0.01,
        epsilon: float = 1e-8,
        selection_method: str = "top_l1",
        adjust_lr: Optional[str] = "spectral_norm",
        ns_coeffs=None,
        seed: int = 0,
        tp_mesh: Optional[DeviceMesh] = None,
    ):
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not (0.0 < fraction <= 1.0):
            raise ValueError(f"Invalid fraction: {fraction}")
        if not (0.0 <= ef_decay <= 1.0):
            raise ValueError(f"Invalid ef_decay: {ef_decay}")
        if selection_method not in ("top_l1", "random"):
            raise ValueError(f"Invalid selection_method: {selection_method}")
        if adjust_lr not in _ADJUST:
            raise ValueError(f"Invalid adjust_lr value: {adjust_lr}")
        defaults = dict(lr=lr, fraction=fraction, ef_decay=ef_decay, beta1=betas[0], beta2=betas[1],
                        weight_decay=weight_decay, epsilon=epsilon, algorithm="dion2", step=0,
                        selection_method=selection_method, adjust_lr=adjust_lr)
        super().__init__(params, defaults)
        if isinstance(distributed_mesh, DeviceMesh):
            if distributed_mesh.ndim != 1:
                raise ValueError("Only 1D DeviceMesh is supported; for HSDP pass the 1D shard sub-mesh.")
            self._rank, self._world, self._pg = (distributed_mesh.get_local_rank(), distributed_mesh.size(),
                                                 distributed_mesh.get_group())
        elif isinstance(distributed_mesh, ProcessGroup):
            self._rank, self._world, self._pg = (dist.get_rank(distributed_mesh),
                                                 dist.get_world_size(distributed_mesh), distributed_mesh)
        else:
            self._rank, self._world, self._pg = 0, 1, None
        self._coeffs = _resolve_coeffs(ns_coeffs)
        # tensor-parallel sub-mesh (FSDP x TP): the selected rows of a matrix are
        # assembled over both meshes before Newton-Schulz
        self._tp_pg = tp_mesh.get_group() if isinstance(tp_mesh, DeviceMesh) and tp_mesh.size() > 1 else None
        self._tp = tp_mesh.size() if self._tp_pg is not None else 1
        self._gen: Optional[torch.Generator] = None
        self._p2p_cache: Dict[Any, Any] = {}
        self._seed = seed

    def _state(self, p: Tensor, algo: str) -> Dict[str, Any]:
        st = self.state[p]
        if not st:
            st["momentum"] = torch.zeros_like(p)
            if algo == "adamw":
                st["variance"] = torch.zeros_like(p)
        return st

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            g["step"] += 1
        for g in self.param_groups:
            algo = g["algorithm"]
            params = [p for p in g["params"] if p.grad is not None]
            if not params:
                continue
            if algo in ("dion2", "dion", "muon"):
                for same in group_by_signature(params).values():
                    with phase("dion2/" + "x".join(str(d) for d in same[0].shape)):
                        self._dion2_group(g, same)
            elif algo in ("adamw", "lion"):
                scalar_update(algo, params, [p.grad for p in params], [self._state(p, algo) for p in params], g)
            else:
                raise ValueError(f"Unknown algorithm: {algo}")
        ops.check_status()
        return loss

    # ------------------------------------------------------------------ selection
    def _tp_dim(self, p: Tensor) -> Optional[int]:
        if self._tp_pg is None or not isinstance(p, DTensor):
            return None
        names = p.device_mesh.mesh_dim_names or ()
        if "tp" not in names:
            return None
        pl = p.placements[names.index("tp")]
        return pl.dim if pl.is_shard() else None

    def _dp_dim(self, p: Tensor) -> Optional[int]:
        """Tensor dim sharded over the FSDP (data-parallel shard) mesh."""
        names = p.device_mesh.mesh_dim_names or ()
        for i, pl in enumerate(p.placements):
            if pl.is_shard() and p.device_mesh.size(i) > 1 and (not names or names[i] != "tp"):
                return pl.dim
        return None

    def _select(self, Mb: Tensor, k: int, method: str, col_groups=()) -> Tensor:
        """Row indices [n, k] (sorted) of each matrix of the batch Mb [n, rows, cols].
        ``col_groups``: process groups the columns are split over; the row
        scores are summed over them so all those ranks pick the same rows."""
        n, rows = Mb.shape[:2]
        if k >= rows:
            return torch.arange(rows, device=Mb.device).expand(n, rows)
        if method == "random":
            if self._gen is None or self._gen.device != Mb.device:
                self._gen = torch.Generator(device=Mb.device).manual_seed(self._seed)
            idx = torch.rand((n, rows), device=Mb.device, generator=self._gen).topk(k, dim=1).indices
        else:
            score = Mb.abs().sum(dim=2, dtype=torch.float32)
            for pg in col_groups:
                dist.all_reduce(score, group=pg)
            idx = score.topk(k, dim=1).indices
        return idx.sort(dim=1).values

    # ------------------------------------------------------------------ update
    def _dion2_group(self, g: Dict[str, Any], params: List[Tensor]) -> None:
        p0 = params[0]
        if p0.ndim != 2:
            raise ValueError("Dion2 expects 2-D matrices; use algorithm='adamw' or 'lion' for other tensors.")
        states = [self._state(p, "dion2") for p in params]
        X = to_local(params)
        G = to_local([p.grad for p in params])
        M = to_local([s["momentum"] for s in states])
        ops.dion_momentum_add_(M, G)
        lr, wd = float(g["lr"]), float(g["weight_decay"])
        adj = _ADJUST[g["adjust_lr"]](lr, p0.shape)
        eps = float(g["epsilon"])
        sharded = isinstance(p0, DTensor) and any(
            pl.is_shard() and p0.device_mesh.size(i) > 1 for i, pl in enumerate(p0.placements))
        if M[0].is_cuda and ops.has_ext() and ops._uniform_matrices(M) and ops._uniform_matrices(X):
            self._dion2_group_kernels(g, p0, X, M, lr, wd, adj, eps, sharded)
            return
        Mb = ops.as_batch(M)
        stacked = Mb is None
        if stacked:
            Mb = torch.stack(M)
        rows = Mb.shape[1]
        k = max(1, int(math.ceil(float(g["fraction"]) * rows)))
        tp_dim = self._tp_dim(p0)
        dp_dim = self._dp_dim(p0) if sharded else None
        col_groups = [pg for pg, d in ((self._tp_pg, tp_dim), (self._pg, dp_dim)) if d == 1 and pg is not None]
        idx = self._select(Mb, k, g["selection_method"], col_groups)       # [n, k]
        gather_idx = idx.unsqueeze(-1).expand(-1, -1, Mb.shape[2])
        sel = Mb.gather(1, gather_idx).to(torch.bfloat16)                   # [n, k, cols]
        if tp_dim is not None and self._world == 1:
            U = self._ns_tp_gathered(sel, tp_dim, eps)
        elif sharded and self._world > 1 and dp_dim is not None:
            U = self._orthogonalize_sharded(sel, eps, tp_dim, dp_dim)
        elif self._pg is not None and self._world > 1:
            U = self._orthogonalize_replicated(sel, eps)
        else:
            U = ops.newton_schulz(sel.contiguous(), self._coeffs, eps, clobber_input=True)
        for x in X:
            x.mul_(1.0 - lr * wd)
        for i, x in enumerate(X):
            x.index_add_(0, idx[i], U[i].to(x.dtype), alpha=-adj)
        decay = float(g["ef_decay"])
        Mb.scatter_(1, gather_idx, Mb.gather(1, gather_idx) * decay)
        if stacked:
            for m, mb in zip(M, Mb.unbind(0)):
                m.copy_(mb)

    def _orthogonalize(self, sel: Tensor, eps: float, p0: Tensor, sharded: bool, tp_dim, dp_dim) -> Tensor:
        if tp_dim is not None and self._world == 1:
            return self._ns_tp_gathered(sel, tp_dim, eps)
        if sharded and self._world > 1 and dp_dim is not None:
            return self._orthogonalize_sharded(sel, eps, tp_dim, dp_dim)
        if self._pg is not None and self._world > 1:
            return self._orthogonalize_replicated(sel, eps)
        return ops.newton_schulz(sel.contiguous(), self._coeffs, eps, clobber_input=True)

    def _dion2_group_kernels(self, g, p0, X, M, lr, wd, adj, eps, sharded) -> None:
        """The update on the package's kernels: L1 row scores, per-matrix top-k,
        gather of the selected rows with their selective decay in the same pass,
        Newton-Schulz, and one row-sparse weight update over every matrix (no
        stacking copy of the momentum, no per-matrix loop)."""
        rows = M[0].shape[0]
        k = max(1, int(math.ceil(float(g["fraction"]) * rows)))
        k = min(k, rows)
        tp_dim = self._tp_dim(p0)
        dp_dim = self._dp_dim(p0) if sharded else None
        col_groups = [pg for pg, d in ((self._tp_pg, tp_dim), (self._pg, dp_dim)) if d == 1 and pg is not None]
        scores = None
        if g["selection_method"] == "random":
            if self._gen is None or self._gen.device != M[0].device:
                self._gen = torch.Generator(device=M[0].device).manual_seed(self._seed)
            scores = torch.rand((len(M), rows), device=M[0].device, generator=self._gen)

        def reduce_scores(sc):
            if scores is None:
                for pg in col_groups:
                    dist.all_reduce(sc, group=pg)

        idx, pos = ops.dion2_select_rows(M, k, scores, reduce_scores)
        sel = ops.dion2_gather_decay_(M, idx, float(g["ef_decay"]))
        U = self._orthogonalize(sel, eps, p0, sharded, tp_dim, dp_dim)
        ops.dion2_update_(X, pos, U, 1.0 - lr * wd, adj)

    def _orthogonalize_replicated(self, sel: Tensor, eps: float) -> Tensor:
        W, r = self._world, self._rank
        n, k, c = sel.shape
        sets = (n + W - 1) // W
        buf = torch.zeros((sets * W, k, c), device=sel.device, dtype=sel.dtype)
        buf[:n] = sel
        mine = buf.view(sets, W, k, c)[:, r].contiguous()
        out = ops.newton_schulz(mine, self._coeffs, eps, clobber_input=True)
        allp = torch.empty((W, sets, k, c), device=sel.device, dtype=sel.dtype)
        dist.all_gather_into_tensor(allp.view(W * sets, k, c), out.contiguous(), group=self._pg)
        return allp.transpose(0, 1).reshape(sets * W, k, c)[:n]

    def _ns_tp_gathered(self, full: Tensor, tp_dim: int, eps: float) -> Tensor:
        """Newton-Schulz of the matrices assembled over the TP mesh: rows are
        stacked (column-parallel weights, tp_dim 0) or columns concatenated
        (row-parallel, tp_dim 1); each rank keeps its block of the result."""
        T = self._tp
        parts = torch.empty((T,) + tuple(full.shape), device=full.device, dtype=full.dtype)
        dist.all_gather_into_tensor(parts.view(T, -1), full.contiguous().view(1, -1), group=self._tp_pg)
        whole = torch.cat(list(parts.unbind(0)), dim=1 + tp_dim).contiguous()
        O = ops.newton_schulz(whole, self._coeffs, eps, clobber_input=True)
        me = dist.get_rank(self._tp_pg)
        w = full.shape[1 + tp_dim]
        return O.narrow(1 + tp_dim, me * w, w).contiguous()

    def _orthogonalize_sharded(self, sel: Tensor, eps: float, tp_dim: Optional[int] = None,
                               dp_dim: int = 0) -> Tensor:
        """The selected block of every shard goes to the matrix owner (one
        all-to-all); the owner stacks the W blocks along the FSDP-sharded dim
        (rows: W*k selected rows; columns: the same k rows, all columns),
        assembles over TP as well when the matrix is also TP-sharded,
        orthogonalises, and the blocks come back."""
        W, r = self._world, self._rank
        n, k, c = sel.shape
        sets = (n + W - 1) // W
        if tp_dim is None and dp_dim == 0 and self._p2p_ok(sel, W):
            return self._orthogonalize_sharded_p2p(sel, eps)
        send = torch.zeros((W, sets, k, c), device=sel.device, dtype=sel.dtype)
        for i in range(n):
            send[i % W, i // W] = sel[i]
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv.view(W, -1), send.view(W, -1), group=self._pg)
        if dp_dim == 0:
            full = recv.permute(1, 0, 2, 3).reshape(sets, W * k, c).contiguous()
        else:
            full = recv.permute(1, 2, 0, 3).reshape(sets, k, W * c).contiguous()
        if tp_dim is not None:
            out = self._ns_tp_gathered(full, tp_dim, eps)
        else:
            out = ops.newton_schulz(full, self._coeffs, eps, clobber_input=True)
        if dp_dim == 0:
            back = out.view(sets, W, k, c).permute(1, 0, 2, 3).contiguous()
        else:
            back = out.view(sets, k, W, c).permute(2, 0, 1, 3).contiguous()
        ret = torch.empty_like(back)
        dist.all_to_all_single(ret.view(W, -1), back.view(W, -1), group=self._pg)
        return torch.stack([ret[i % W, i // W] for i in range(n)])

    # ---- in-kernel row exchange over symmetric peer memory
    def _p2p_ok(self, sel: Tensor, W: int) -> bool:
        from ..parallel.symm import p2p_enabled

        n, k, c = sel.shape
        return (W > 1 and self._pg is not None and p2p_enabled(self._pg, sel.device) and c % 8 == 0
                and (W * k) % 8 == 0)

    def _orthogonalize_sharded_p2p(self, sel: Tensor, eps: float) -> Tensor:
        """The selected rows go straight into the owner's [sets, W*k, cols]
        buffer (peer stores, next ranks first), one device barrier, the owner
        orthogonalises, the last Newton-Schulz GEMM stores each rank's k rows
        into that rank's return buffer, one more barrier."""
        from ..parallel.symm import cached_for_heap, heap_for

        W, me = self._world, self._rank
        n, k, c = sel.shape
        sets = (n + W - 1) // W
        blk = k * c * 2
        mat = W * blk
        gather_off, ret_off = 0, sets * mat
        heap = heap_for(self._pg, 2 * sets * mat, "dion2", sel.device)
        key = (heap.uid, n, k, c)

        def build():
            dsts = [heap.ptr_tensor([heap.addr(i % W, gather_off + (i // W) * mat + me * blk)]) for i in range(n)]
            ptrs = heap.ptr_tensor([heap.addr(j, ret_off + (me * sets + s_) * blk) for s_ in range(sets)
                                    for j in range(W)])
            return dsts, ptrs

        dsts, ptrs = cached_for_heap(self._p2p_cache, heap, key, build)
        full = heap.view(gather_off, (sets, W * k, c), torch.bfloat16)
        for i in range(n, sets * W):
            if i % W == me:  # this rank owns an absent matrix of the last set
                full[i // W].zero_()
        sel = sel.contiguous()
        for t in range(n):
            i = (me + 1 + t) % n if n > 1 else t  # next ranks' matrices first
            heap.push(sel[i], dsts[i])
        heap.barrier()
        ops.newton_schulz(full, self._coeffs, eps, clobber_input=False, out_ptrs=ptrs, rows_per_ptr=k,
                          rot_rows=((me + 1) % W) * k)
        heap.barrier()
        ret = heap.view(ret_off, (W, sets, k, c), torch.bfloat16)
        return torch.stack([ret[i % W, i // W] for i in range(n)])

