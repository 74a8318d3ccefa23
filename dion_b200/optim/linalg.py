"""Orthogonalisation for Dion's power iteration.

``orthogonalize(P)`` for a batch of fp32 matrices P (b, d, r):
  * d <= r : QR of P (reduced Q);
  * d >  r : randomised Cholesky QR (the reference's "rcqr",
    ada_dion/optim/adadion_v2.py:1645-1685):
        S ~ N(0, 1/k), k = ceil(oversample*r/128)*128
        R1 = qr(S P).R ;  P = P R1^-1
        R2 = chol(P^T P) ;  P = P R2^-1
The big products (S P, P R^-1, P^T P) run on the tcgen05 tensor cores
(tf32, fp32 accumulate); the r x r / k x r factorisations use the package's
sm_100a kernels when present and torch.linalg otherwise.

``distributed_orthogonalize`` is the inner-sharded (TP) variant
(adadion_v2.py:1690-1790): rows of P are split across the inner mesh, the
sketch S P and the Gram P^T P are reduce-scattered so each rank factors one
matrix of the batch, and the triangular factors are all-gathered.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor, Replicate, Shard

from .. import ops

__all__ = ["orthogonalize", "distributed_orthogonalize", "sketch_size", "tri_inv_upper", "cholesky_upper"]


def sketch_size(r: int, oversample: float) -> int:
    return int(math.ceil(oversample * r / 128.0) * 128)


def tri_inv_upper(R: Tensor) -> Tensor:
    """Inverse of a batch of upper-triangular matrices (fp32)."""
    if R.is_cuda and ops.has_ext() and hasattr(ops.ext(), "tri_inv_upper"):
        out = torch.empty_like(R)
        ops.ext().tri_inv_upper(R.contiguous(), out)
        return out
    eye = torch.eye(R.size(-1), device=R.device, dtype=R.dtype).expand_as(R)
    return torch.linalg.solve_triangular(R, eye, upper=True)


def cholesky_upper(A: Tensor) -> Tensor:
    """Upper Cholesky factor of a batch of SPD matrices (fp32); non-SPD
    entries give NaN/garbage that the Dion guard later zeroes."""
    if A.is_cuda and ops.has_ext() and hasattr(ops.ext(), "cholesky_upper"):
        out = torch.empty_like(A)
        ops.ext().cholesky_upper(A.contiguous(), out)
        return out
    R, _ = torch.linalg.cholesky_ex(A, upper=True)
    return R


def qr_r(A: Tensor) -> Tensor:
    """R factor of the QR decomposition of a batch of tall matrices (fp32)."""
    if A.is_cuda and ops.has_ext() and hasattr(ops.ext(), "qr_r"):
        out = torch.empty(A.size(0), A.size(-1), A.size(-1), device=A.device, dtype=A.dtype)
        ops.ext().qr_r(A.contiguous(), out)
        return out
    return torch.linalg.qr(A, mode="r")[1]


def _right_solve(P: Tensor, R: Tensor) -> Tensor:
    """P R^-1 for upper-triangular R: invert the r x r factor, then one GEMM."""
    if P.is_cuda:
        Rinv = tri_inv_upper(R)
        return ops.matmul(P, Rinv)
    return torch.linalg.solve_triangular(R, P, upper=True, left=False)


def orthogonalize(P: Tensor, oversample: float = 1.25, generator: Optional[torch.Generator] = None) -> Tensor:
    assert P.ndim == 3, "Expected a batch of matrices"
    dtype = P.dtype
    Pf = P.float().contiguous()
    b, d, r = Pf.shape
    if d <= r:
        Q, _ = torch.linalg.qr(Pf)
        return Q.to(dtype)
    k = sketch_size(r, oversample)
    S = torch.randn((b, k, d), device=P.device, dtype=torch.float32, generator=generator)
    S.mul_(math.sqrt(1.0 / k))
    SP = ops.matmul(S, Pf) if P.is_cuda else S @ Pf
    R1 = qr_r(SP)
    Pf = _right_solve(Pf, R1)
    PP = ops.matmul(Pf.transpose(1, 2), Pf, symmetric=True) if P.is_cuda else Pf.mT @ Pf
    R2 = cholesky_upper(PP)
    Pf = _right_solve(Pf, R2)
    return Pf.to(dtype)


def distributed_orthogonalize(P: DTensor, oversample: float = 1.25, shard_mesh_dim: Optional[int] = None) -> DTensor:
    """Orthogonalise a batch of row-sharded DTensor matrices (see module doc)."""
    assert isinstance(P, DTensor)
    assert P.ndim >= 3
    dtype = P.dtype
    orig = P.placements
    full_rep = [Replicate() for _ in orig]
    batch_sharded = list(full_rep)
    if shard_mesh_dim is not None:
        batch_sharded[shard_mesh_dim] = Shard(0)
    mesh = P.device_mesh
    d, r = P.shape[-2:]
    if d <= r:
        single = P.redistribute(placements=batch_sharded)
        Q, _ = torch.linalg.qr(single.to_local().float(), mode="reduced")
        out = DTensor.from_local(Q.to(dtype).contiguous(), mesh, single.placements, run_check=False,
                                 shape=single.shape, stride=single.stride())
        return out.redistribute(placements=orig)
    k = sketch_size(r, oversample)
    P_local = P.to_local().float().contiguous()
    S_local = torch.randn((P_local.size(0), k, P_local.size(1)), device=P_local.device) * math.sqrt(1.0 / k)
    SP_local = ops.matmul(S_local, P_local) if P_local.is_cuda else S_local @ P_local
    sp_pl = [pl if not (pl.is_shard() and pl.dim == P.ndim - 2) else None for pl in orig]
    from torch.distributed.tensor import Partial

    sp_pl = [Partial() if x is None else x for x in sp_pl]
    SP = DTensor.from_local(SP_local, mesh, sp_pl, run_check=False)
    SP_single = SP.redistribute(placements=batch_sharded)
    R_local = qr_r(SP_single.to_local().float().contiguous())
    R = DTensor.from_local(R_local, mesh, SP_single.placements, run_check=False).redistribute(placements=full_rep)
    P_local = _right_solve(P_local, R.to_local().contiguous())
    PP_local = ops.matmul(P_local.transpose(1, 2), P_local, symmetric=True) if P_local.is_cuda else P_local.mT @ P_local
    PP = DTensor.from_local(PP_local, mesh, sp_pl, run_check=False)
    PP_single = PP.redistribute(placements=batch_sharded)
    R2_local = cholesky_upper(PP_single.to_local().contiguous())
    R2 = DTensor.from_local(R2_local, mesh, PP_single.placements, run_check=False).redistribute(placements=full_rep)
    P_local = _right_solve(P_local, R2.to_local().contiguous())
    return DTensor.from_local(P_local.to(dtype).contiguous(), mesh, orig, run_check=False, shape=P.shape,
                              stride=P.stride())
